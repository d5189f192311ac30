"""The CUDA device's generated row-chain kernels, run on the CPU (RGC_ROW_CHAINS=1).

For each chain of a plan, the device library describes the kernel it generates (its source and
the slots, periods and broadcast descriptors bound to its parameters). The source is compiled
for the host with tests/row_emulator/shim.h, which runs every CUDA thread of a block as an OS
thread with real barriers and warp exchanges, and executed on the CPU interpreter's slots as
they are just before the chain. Every value the kernel stores must equal, bit for bit, what the
interpreter computes by running the chain's steps one by one: the same operations in the same
order, sums in rg's fast_sum order, maxima and minima as rg's sequential fold. (The host's libm
is glibc's, as the interpreter's is, so exp and tanh agree too; on the GPU they are CUDA's.)
"""
import ctypes
import json
import os
import subprocess

import numpy as np
import pytest

import rustautograd_b200
from rustautograd_b200 import frontend as F

HERE = os.path.dirname(os.path.abspath(__file__))
NP = {"float32": np.float32, "float64": np.float64, "int32": np.int32}


class FDiv(ctypes.Structure):
    _fields_ = [("d", ctypes.c_uint), ("m", ctypes.c_uint), ("s", ctypes.c_uint)]


class FDims(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int), ("d", FDiv * 8), ("st", ctypes.c_longlong * 8)]


class ElemArgs(ctypes.Structure):
    _fields_ = [("n", ctypes.c_longlong), ("vec", ctypes.c_int), ("small", ctypes.c_int), ("out", ctypes.c_void_p * 64),
                ("inp", ctypes.c_void_p * 64), ("row", FDiv * 64), ("bc", ctypes.c_void_p), ("bc64", ctypes.c_void_p)]


DRIVER = """
extern "C" void rg_emulate(const ElemArgs* a, int grid) {
  gridDim.x = (unsigned)grid;
  blockDim.x = 256;
  for (int b = 0; b < grid; ++b) {
    RgBlock blk;
    rg_block = &blk;
    std::vector<std::thread> ts;
    for (int t = 0; t < 256; ++t)
      ts.emplace_back([a, b, t] {
        threadIdx.x = (unsigned)t;
        blockIdx.x = (unsigned)b;
        KERNEL(*a);
      });
    for (auto& th : ts) th.join();
  }
}
"""


@pytest.fixture(autouse=True)
def _chains(oracle, monkeypatch):
    monkeypatch.setenv("RGC_ROW_CHAINS", "1")
    F.use(oracle, "cpu")
    yield


def run_chain_kernels(oracle, tmp_path, fn, args):
    """Emulates every row-chain kernel of fn's device plan; returns how many ran."""
    c = F.compile(fn, args, validate="none", device="cuda-plan")
    blob = c._n.plan_blob()
    leaves = [F.tensor(x) for x in F.flatten(args)[0]]
    inputs = [(x.numpy().tobytes(), list(x.shape), x.dtype) for x in leaves]
    lib = ctypes.CDLL(rustautograd_b200.LIBRARY)
    lib.rgc_debug_row_kernel.restype = ctypes.c_int
    chains = json.loads(c._n.row_chains())
    ran = 0
    for index in range(len(chains)):
        buf = ctypes.create_string_buffer(1 << 20)
        src = tmp_path / f"k{index}.cu"
        rc = lib.rgc_debug_row_kernel(blob, len(blob), index, buf, len(buf), str(src).encode())
        assert rc in (0, 1), buf.value.decode()
        if rc == 1:
            continue
        info = json.loads(buf.value.decode())
        before = oracle.plan_blob_slots(blob, inputs, list(range(info["first"])) + info["before"])
        after = oracle.plan_blob_slots(blob, inputs, list(range(info["last"] + 1)))
        mem = {}

        def slot(s):
            if s not in mem:
                data, dt = before[s]
                mem[s] = np.frombuffer(bytearray(data), dtype=NP[dt]).copy()
            return mem[s]
        a = ElemArgs()
        a.n = info["rows"]
        for k, s in enumerate(info["in_slots"]):
            a.inp[k] = slot(s).ctypes.data
            a.row[k] = FDiv(*info["in_div"][k])
        for q, s in enumerate(info["out_slots"]):
            a.out[q] = slot(s).ctypes.data
        bcs = (FDims * max(1, len(info["bcs"])))()
        for i, b in enumerate(info["bcs"]):
            bcs[i].rank = b["rank"]
            for q in range(8):
                bcs[i].d[q] = FDiv(*b["d"][q])
                bcs[i].st[q] = b["st"][q]
        a.bc = ctypes.addressof(bcs)
        code = "\n".join(line for line in src.read_text().splitlines() if "griddepcontrol" not in line)
        wrapper = tmp_path / f"emu{index}.cpp"
        wrapper.write_text('#include <math.h>\n#include "shim.h"\n' + code + f"\n#define KERNEL {info['name']}\n" + DRIVER)
        so = tmp_path / f"emu{index}.so"
        subprocess.run(["g++", "-O1", "-std=c++17", "-ffp-contract=off", "-fPIC", "-shared", "-w", "-I", os.path.join(HERE, "row_emulator"),
                        str(wrapper), "-o", str(so), "-lpthread"], check=True)
        emu = ctypes.CDLL(str(so))
        blocks = (info["rows"] + info["rows_per_block"] - 1) // info["rows_per_block"]
        emu.rg_emulate(ctypes.byref(a), ctypes.c_int(min(2, blocks)))
        for s in info["out_slots"]:
            want = np.frombuffer(after[s][0], dtype=mem[s].dtype)
            got = mem[s]
            assert got.tobytes() == want.tobytes(), (index, s, info["members"], np.flatnonzero(got.view(np.uint8) != want.view(np.uint8))[:10])
        ran += 1
    return ran


def test_gpt_step_row_kernels(oracle, tmp_path):
    model = F.gpt.GPT(vocab=24, block=16, d=32, heads=4, layers=1)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 24, size=500, dtype="int32"))
    assert run_chain_kernels(oracle, tmp_path, F.gpt.make_train_step(model, opt, 6), (state, tokens)) >= 6


@pytest.mark.parametrize("dtype,cols", [("float32", 10), ("float32", 6), ("float64", 12), ("float64", 7)])
def test_softmax_layernorm_row_kernels(oracle, tmp_path, dtype, cols):
    """Rows that are not a multiple of the vector width (scalar path), shorter than eight (the
    fast_sum tail only), and f64."""
    rng = np.random.default_rng(cols)
    x = F.tensor(rng.normal(size=(37, cols)).astype(dtype))
    g = F.tensor(rng.normal(size=(cols,)).astype(dtype))
    mask = F.tensor((rng.random((37, cols)) > 0.3).astype(dtype))

    def f(x, g, mask):
        z = F.where(mask, x * 3.0, -1e9)
        p = F.nn.softmax(z)
        mu = x.mean(axis=-1, keepdims=True)
        v = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
        y = (x - mu) / (v + 1e-5).sqrt() * g
        return (p * y).sum() + F.nn.log_softmax(y).min()
    assert run_chain_kernels(oracle, tmp_path, F.value_and_grad(f, argnums=(0, 1)), (x, g, mask)) >= 2


def test_signed_zero_ties_and_nan_rows(oracle, tmp_path):
    """Row maxima and minima over rows with -0 and +0 ties, NaN and infinities: the kernel's
    combination of eight lanes equals rg's sequential fold bit for bit."""
    vals = np.array([[0.0, -0.0, -1.0, 0.0, -0.0, -2.0, -0.0, -3.0, 0.0, -0.0, -4.0],
                     [-0.0, 0.0, -0.0, 0.0, -0.0, 0.0, -0.0, 0.0, -0.0, 0.0, -0.0],
                     [1.0, np.nan, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0, 10.0],
                     [-np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf, -np.inf],
                     [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, -0.0]], dtype="float32")
    x = F.tensor(np.concatenate([vals, -vals]))

    def f(x):
        hi = x.max(axis=-1, keepdims=True)
        lo = x.min(axis=-1, keepdims=True)
        return (x * 2.0 + hi).sum(axis=-1, keepdims=True) + lo * 1.0, hi, lo
    assert run_chain_kernels(oracle, tmp_path, f, (x,)) >= 1


def test_periodic_and_broadcast_inputs(oracle, tmp_path):
    """A (T, C) table repeated over the batch (periodic), a (B, 1, C) tensor broadcast over T
    (strided), and a per-row statistic read back by the full pass."""
    rng = np.random.default_rng(7)
    x = F.tensor(rng.normal(size=(3, 5, 16)).astype("float32"))
    pos = F.tensor(rng.normal(size=(5, 16)).astype("float32"))
    scale = F.tensor(rng.normal(size=(3, 1, 16)).astype("float32"))

    def f(x, pos, scale):
        h = x + pos
        m = h.max(axis=-1, keepdims=True)
        e = F.exp(h - m) * scale
        return e / e.sum(axis=-1, keepdims=True)
    assert run_chain_kernels(oracle, tmp_path, f, (x, pos, scale)) >= 1
