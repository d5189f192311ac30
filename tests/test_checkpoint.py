"""Checkpoints (the safetensors layout of python/rg/checkpoint.py) and sessions whose state stays
in one exec between runs, on the CPU oracle: round trips, the file layout itself, metadata,
rejection of mismatched files, and save / restore / continue equal to one uninterrupted run."""
import json
import struct

import numpy as np
import pytest

from rustautograd_b200 import frontend as F


@pytest.fixture(autouse=True)
def _cpu(oracle):
    F.use(oracle, "cpu")
    yield


def test_save_and_load_a_tree_with_metadata(tmp_path):
    tree = {"w": F.tensor(np.arange(6, dtype="float32").reshape(2, 3)), "b": [F.tensor(np.array([1.5, -2.0])), F.tensor(np.array([7], "int32"))]}
    path = str(tmp_path / "t.safetensors")
    F.checkpoint.save(path, tree, {"note": "hello"})
    back, meta = F.checkpoint.load(path, with_metadata=True)
    assert meta == {"note": "hello"}
    for a, b in zip(F.tree_leaves(tree), F.tree_leaves(back)):
        assert a.dtype == b.dtype and np.array_equal(a.numpy(), b.numpy())
    # The layout: header length, JSON header with dotted names and data offsets, raw bytes.
    raw = open(path, "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    assert header["w"] == {"dtype": "F32", "shape": [2, 3], "data_offsets": [header["w"]["data_offsets"][0], header["w"]["data_offsets"][0] + 24]}
    assert set(header) == {"b.0", "b.1", "w", "__metadata__"}
    w0 = header["w"]["data_offsets"][0]
    np.testing.assert_array_equal(np.frombuffer(raw[8 + n + w0:8 + n + w0 + 24], "float32"), np.arange(6))


def test_corrupt_or_foreign_files(tmp_path):
    path = str(tmp_path / "bad.safetensors")
    open(path, "wb").write(b"\x01\x02")
    with pytest.raises(ValueError):
        F.checkpoint.load(path)
    # A file without rg's tree metadata loads as a flat dict.
    hdr = json.dumps({"x": {"dtype": "F64", "shape": [2], "data_offsets": [0, 16]}}).encode()
    open(path, "wb").write(struct.pack("<Q", len(hdr)) + hdr + np.array([1.0, 2.0]).tobytes())
    assert list(F.checkpoint.load(path)) == ["x"]


def _linreg():
    x = np.random.default_rng(0).normal(size=(64, 4)).astype("float32")
    y = x @ np.arange(4, dtype="float32")

    def step(s, b):
        value, g = F.value_and_grad(lambda w, b: (((b[0] @ w) - b[1]) ** 2).mean())(s["w"], b)
        return {"w": s["w"] - 0.05 * g, "n": s["n"] + 1.0}, value
    state = {"w": F.zeros(4), "n": F.tensor(0.0)}
    data = [F.tensor(x), F.tensor(y)]
    return step, state, data


def test_session_save_restore_continue_equals_one_run(tmp_path):
    step, state, data = _linreg()
    c = F.compile(step, (state, data), validate="none", device="cpu")
    full = F.run(c, state, data, steps=30)
    s = F.Session(c, state, data)
    h1 = s.run(12).history["aux"]
    path = str(tmp_path / "s.safetensors")
    s.save(path, {"step": "12"})
    s2 = F.Session(c, state, data)
    s2.restore(path)
    h2 = s2.run(18).history["aux"]
    assert list(h1) + list(h2) == list(full.history["aux"])
    np.testing.assert_array_equal(s2.state["w"].numpy(), full.state["w"].numpy())
    # The session's checkpoint is an ordinary checkpoint of the state tree.
    tree, meta = F.checkpoint.load(path, with_metadata=True)
    assert meta == {"step": "12"} and float(tree["n"]) == 12.0


def test_restore_rejects_another_state_structure(tmp_path):
    step, state, data = _linreg()
    c = F.compile(step, (state, data), validate="none", device="cpu")
    path = str(tmp_path / "other.safetensors")
    F.checkpoint.save(path, {"w": F.zeros(5), "n": F.tensor(0.0)})
    with pytest.raises(ValueError):
        F.Session(c, state, data).restore(path)
