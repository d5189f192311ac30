"""Row chains on the CUDA device (on by default; RGC_ROW_CHAINS=0 turns them off): the same plans
with and without chains give bit-identical results, since a chain evaluates the same operations
in the same order as the plan's own kernels; rows without transcendental functions also equal
the CPU interpreter's. (The generated kernels are also checked on the CPU, thread by thread
against the interpreter, by test_row_kernels_emulated.py.)
"""
import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import assert_bits_equal, compile_and_compare

pytestmark = pytest.mark.gpu


def outputs(fn, args, chains, monkeypatch):
    monkeypatch.setenv("RGC_ROW_CHAINS", "1" if chains else "0")
    c = F.compile(fn, args, validate="none", device="cuda")
    leaves = [F.tensor(x) for x in F.flatten(args)[0]]
    return [F.Tensor(t).numpy() for t in c._n.call([t._t for t in leaves])], c


def gpt(d=64, heads=4, layers=2, block=32, batch=16):
    model = F.gpt.GPT(vocab=48, block=block, d=d, heads=heads, layers=layers)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 48, size=5000, dtype="int32"))
    return F.gpt.make_train_step(model, opt, batch), (state, tokens)


@pytest.mark.parametrize("cfg", [dict(), dict(d=128, heads=4, block=128, batch=8, layers=1)])
def test_gpt_step_identical_with_and_without_row_chains(cuda, monkeypatch, cfg):
    F.use(cuda, "cuda")
    fn, args = gpt(**cfg)
    on, _ = outputs(fn, args, True, monkeypatch)
    off, _ = outputs(fn, args, False, monkeypatch)
    for k, (a, b) in enumerate(zip(on, off)):
        assert_bits_equal(a, b, f"output {k}")


@pytest.mark.parametrize("dtype,cols", [("float32", 256), ("float32", 10), ("float64", 96), ("float64", 7)])
def test_softmax_layernorm_identical_with_and_without_row_chains(cuda, monkeypatch, dtype, cols):
    F.use(cuda, "cuda")
    rng = np.random.default_rng(cols)
    x = F.tensor(rng.normal(size=(300, cols)).astype(dtype))
    g = F.tensor(rng.normal(size=(cols,)).astype(dtype))
    mask = F.tensor((rng.random((300, cols)) > 0.3).astype(dtype))

    def f(x, g, mask):
        p = F.nn.softmax(F.where(mask, x * 3.0, -1e9))
        mu = x.mean(axis=-1, keepdims=True)
        y = (x - mu) / (((x - mu) ** 2).mean(axis=-1, keepdims=True) + 1e-5).sqrt() * g
        return (p * y).sum() + F.nn.log_softmax(y).min()
    fn = F.value_and_grad(f, argnums=(0, 1))
    on, _ = outputs(fn, (x, g, mask), True, monkeypatch)
    off, _ = outputs(fn, (x, g, mask), False, monkeypatch)
    for k, (a, b) in enumerate(zip(on, off)):
        assert_bits_equal(a, b, f"output {k}")


def test_row_extrema_equal_the_interpreter(cuda, oracle, monkeypatch):
    """Maxima and minima over rows with -0/+0 ties, NaN and infinities, and a sum: no
    transcendental function, so the device equals the CPU interpreter bit for bit."""
    monkeypatch.setenv("RGC_ROW_CHAINS", "1")
    F.use(cuda, "cuda")
    rng = np.random.default_rng(3)
    x = rng.normal(size=(512, 40)).astype("float32")
    x[::7, ::3] = 0.0
    x[1::7, ::5] = -0.0
    x[2::97, 4] = np.nan
    x[3::89, :] = -np.inf
    t = F.tensor(x)

    def f(x):
        hi = x.max(axis=-1, keepdims=True)
        lo = x.min(axis=-1, keepdims=True)
        return (x * 2.0 + hi).sum(axis=-1, keepdims=True) + lo, hi, lo
    gpu, cpu, _ = compile_and_compare(oracle, f, (t,))
    for k, (a, b) in enumerate(zip(gpu, cpu)):
        assert_bits_equal(a, b, f"output {k}")
