"""The device's fused-attention rewrite (every match with RGC_FUSED_ATTENTION=1; by default only
the shapes where the device's fused kernels are faster), on the CPU: plans
built for the CUDA device through the oracle's "cuda-plan" device, whose interpreter runs the fused
ops' CPU definition, against rg's own plan of the same graph.

The fused ops sum the softmax and its gradient in another order than rg's chain of ops, so values
agree to rounding (1e-4, max-norm), not bit for bit. A gradient that is zero in exact arithmetic
(the key bias of an attention layer) is rounding noise on both sides and is not compared.
"""
import json
import math

import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from rustautograd_b200.frontend import nn


@pytest.fixture(autouse=True)
def _frontend(oracle, monkeypatch):
    F.use(oracle, "cpu")
    monkeypatch.setenv("RGC_FUSED_ATTENTION", "1")
    yield


def ops_of(c):
    return [p.get("op") for p in json.loads(c._n.plan_summary()) if "op" in p]


def both(fn, args):
    out = {}
    for dev in ("cpu", "cuda-plan"):
        c = F.compile(fn, args, validate="none", device=dev)
        leaves = [F.tensor(x) for x in F.flatten(args)[0]]
        out[dev] = ([F.Tensor(g).numpy() for g in c._n.call([t._t for t in leaves])], c)
    return out


def rel(a, b):
    a = a.astype(np.float64)
    return float(np.abs(a - b).max()) / max(float(np.abs(a).max()), 1e-30)


def attention(q, k, v, mask):
    scores = q @ F.swapaxes(k, -1, -2) / math.sqrt(q.shape[-1])
    scores = F.where(mask, scores, -1e9)
    return nn.softmax(scores) @ v


@pytest.mark.parametrize("shape", [(2, 3, 16, 8), (1, 4, 33, 5), (3, 7, 4)])
def test_attention_values_and_gradients_match_rgs_plan(shape):
    rng = np.random.default_rng(7)
    q, k, v, w = (F.tensor(rng.normal(size=shape).astype("float32")) for _ in range(4))
    mask = F.tril(shape[-2])

    def fn(q, k, v, w):
        return F.value_and_grad(lambda q, k, v: (attention(q, k, v, mask) * w).sum(), argnums=(0, 1, 2))(q, k, v)
    out = both(fn, (q, k, v, w))
    assert ops_of(out["cuda-plan"][1]).count("attention") == 1
    assert ops_of(out["cuda-plan"][1]).count("attention_grad") == 1
    assert "attention" not in ops_of(out["cpu"][1])
    for k_, (a, b) in enumerate(zip(out["cpu"][0], out["cuda-plan"][0])):
        assert rel(a, b) <= 1e-4, f"output {k_}"


def test_forward_only_attention_is_left_alone():
    """Without the backward pattern (no gradient) nothing is rewritten."""
    rng = np.random.default_rng(8)
    q, k, v = (F.tensor(rng.normal(size=(2, 8, 4)).astype("float32")) for _ in range(3))
    out = both(lambda q, k, v: attention(q, k, v, F.tril(8)), (q, k, v))
    assert "attention" not in ops_of(out["cuda-plan"][1])
    assert rel(out["cpu"][0][0], out["cuda-plan"][0][0]) == 0.0


def test_gpt_step_with_fused_attention_matches_rgs_plan():
    model = F.gpt.GPT(vocab=32, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 32, size=2000, dtype="int32"))
    out = both(F.gpt.make_train_step(model, opt, 8), (state, tokens))
    ops = ops_of(out["cuda-plan"][1])
    assert ops.count("attention") == 2 and ops.count("attention_grad") == 2  # one pair per layer
    d = 32
    for k_, (a, b) in enumerate(zip(out["cpu"][0], out["cuda-plan"][0])):
        if a.dtype.kind != "f":
            assert np.array_equal(a, b), f"output {k_}"
        elif a.shape == (3 * d,):
            # The fused q/k/v bias and its optimizer state: the key third is rounding noise.
            keep = np.r_[0:d, 2 * d:3 * d]
            assert rel(a[keep], b[keep]) <= 1e-4, f"output {k_}"
        else:
            assert rel(a, b) <= 1e-4, f"output {k_}"


def test_default_fuses_the_shapes_measured_faster(monkeypatch):
    """By default the device fuses attention of length 128 or 256 with head size 32, and of
    length 256 with head size 64 (measured faster on a B200), and leaves other shapes (length
    128 with head size 64 among them) to the unfused plan; RGC_FUSED_ATTENTION=0 turns fusion off
    for every shape."""
    monkeypatch.delenv("RGC_FUSED_ATTENTION", raising=False)
    rng = np.random.default_rng(9)

    def plan(shape):
        q, k, v, w = (F.tensor(rng.normal(size=shape).astype("float32")) for _ in range(4))
        mask = F.tril(shape[-2])
        fn = lambda q, k, v, w: F.value_and_grad(lambda q, k, v: (attention(q, k, v, mask) * w).sum(), argnums=(0, 1, 2))(q, k, v)
        return ops_of(F.compile(fn, (q, k, v, w), validate="none", device="cuda-plan"))
    assert "attention" not in plan((2, 8, 4))
    assert "attention" not in plan((1, 2, 128, 64))
    assert "attention" in plan((1, 2, 128, 32))
    assert "attention" in plan((1, 1, 256, 32))
    assert "attention" in plan((1, 1, 256, 64))
    monkeypatch.setenv("RGC_FUSED_ATTENTION", "0")
    assert "attention" not in plan((1, 2, 128, 32))


def test_gpt_step_at_tensor_core_shapes_uses_the_packed_form():
    """At length 128 with head size 32 the fused ops read q, k, v straight from the (B, T, 3, H, d)
    projection output and give the gradient of that tensor: no head-split transpose, no
    q / k / v slices, no concat or transpose of the gradients. Values against rg's plan as above."""
    model = F.gpt.GPT(vocab=32, block=128, d=64, heads=2, layers=1)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 32, size=2000, dtype="int32"))
    out = both(F.gpt.make_train_step(model, opt, 2), (state, tokens))
    steps = [p for p in json.loads(out["cuda-plan"][1]._n.plan_summary()) if "op" in p]
    fwd = [p for p in steps if p["op"] == "attention"]
    bwd = [p for p in steps if p["op"] == "attention_grad"]
    assert len(fwd) == 1 and len(bwd) == 1
    assert fwd[0]["args"][0] == [2, 128, 3, 2, 32] and bwd[0]["shape"] == [2, 128, 3, 2, 32]
    assert not [p for p in steps if p["op"] in ("transpose", "concat") and 3 in p["shape"][:1]]
    d = 64
    for k_, (a, b) in enumerate(zip(out["cpu"][0], out["cuda-plan"][0])):
        if a.dtype.kind != "f":
            assert np.array_equal(a, b), f"output {k_}"
        elif a.shape == (3 * d,):
            keep = np.r_[0:d, 2 * d:3 * d]
            assert rel(a[keep], b[keep]) <= 1e-4, f"output {k_}"
        else:
            assert rel(a, b) <= 1e-4, f"output {k_}"


def _packed_layer_with_mask(mask_np):
    """A GPT attention layer (projection, head split, attention, head merge, projection) over a
    given (T, T) mask, its value and gradients for inputs and weights."""
    rng = np.random.default_rng(11)
    b, t, d, heads = 2, mask_np.shape[0], 64, 2
    mk = lambda *s: F.tensor((rng.normal(size=s) * 0.3).astype("float32"))
    p = {"qkv": {"w": mk(d, 3 * d), "b": mk(3 * d)}, "out": {"w": mk(d, d), "b": mk(d)}}
    x, w = mk(b, t, d), mk(b, t, d)
    mask = F.tensor(mask_np)

    def fn(p, x, w):
        return F.value_and_grad(lambda p, x: (F.gpt.attention(p, x, heads, mask) * w).sum(), argnums=(0, 1))(p, x)
    return fn, (p, x, w)


def general_mask(t=128, seed=5):
    m = (np.random.default_rng(seed).random((t, t)) < 0.6).astype("float32")
    np.fill_diagonal(m, 1.0)
    m[3] = 0.0  # a row with every key masked
    return m


def test_packed_form_with_a_general_mask_matches_rgs_plan():
    """The packed form with a mask that is not causal (packed into bits by the kernels, and a
    fully masked row) against rg's plan; the key bias's gradient is left out as above."""
    fn, args = _packed_layer_with_mask(general_mask())
    out = both(fn, args)
    steps = [p for p in json.loads(out["cuda-plan"][1]._n.plan_summary()) if "op" in p]
    assert [p["args"][0] for p in steps if p["op"] == "attention"] == [[2, 128, 3, 2, 32]]
    for k_, (a, b) in enumerate(zip(out["cpu"][0], out["cuda-plan"][0])):
        if a.shape == (3 * 64,):
            keep = np.r_[0:64, 128:192]
            assert rel(a[keep], b[keep]) <= 1e-4, f"output {k_}"
        else:
            assert rel(a, b) <= 1e-4, f"output {k_}"
