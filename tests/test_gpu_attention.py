"""The device's fused attention kernels (attention.cu) against the CPU oracle running the very
same plan blob (its attn_fwd / attn_bwd definitions), and against the device's unfused plan of
the same graph.

Shapes: small ones (T not 128 or 256, or head sizes other than 32 and 64) run on CUDA cores;
T = 128 and 256 with head sizes 32 and 64 (configs 4 and 5) run on the tensor cores. The bound
is 1e-4 (max-norm relative), as for every fp32 value that passes through exp: the fused kernels
sum the softmax and its gradient in another order than the plan's chain of ops.
"""
import json
import math

import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from rustautograd_b200.frontend import nn
from helpers import max_rel, np_of, triple

pytestmark = pytest.mark.gpu


def attention(q, k, v, mask):
    scores = F.where(mask, q @ F.swapaxes(k, -1, -2) / math.sqrt(q.shape[-1]), -1e9)
    return nn.softmax(scores) @ v


def ops_of(c):
    return [p.get("op") for p in json.loads(c._n.plan_summary()) if "op" in p]


def run(fn, args, fused, monkeypatch):
    monkeypatch.setenv("RGC_FUSED_ATTENTION", "1" if fused else "0")
    c = F.compile(fn, args, validate="none", device="cuda")
    leaves = [F.tensor(x) for x in F.flatten(args)[0]]
    return [F.Tensor(t).numpy() for t in c._n.call([t._t for t in leaves])], c, leaves


@pytest.mark.parametrize("shape", [(2, 3, 16, 8), (1, 2, 33, 5), (2, 4, 128, 32), (2, 2, 256, 64), (1, 3, 256, 32), (1, 2, 128, 64)])
def test_fused_attention_matches_the_oracle_and_the_unfused_plan(cuda, oracle, monkeypatch, shape):
    F.use(cuda, "cuda")
    rng = np.random.default_rng(sum(shape))
    q, k, v, w = (F.tensor(rng.normal(size=shape).astype("float32")) for _ in range(4))
    mask = F.tril(shape[-2])

    def fn(q, k, v, w):
        return F.value_and_grad(lambda q, k, v: (attention(q, k, v, mask) * w).sum(), argnums=(0, 1, 2))(q, k, v)
    fused, c, leaves = run(fn, (q, k, v, w), True, monkeypatch)
    assert ops_of(c).count("attention") == 1 and ops_of(c).count("attention_grad") == 1
    cpu = [np_of(x) for x in oracle.run_plan_blob(c.plan_blob(), [triple(t) for t in leaves])]
    plain, c0, _ = run(fn, (q, k, v, w), False, monkeypatch)
    assert "attention" not in ops_of(c0)
    for n, (g, o, u) in enumerate(zip(fused, cpu, plain)):
        assert max_rel(g, o) <= 1e-4, f"output {n} against the oracle: {max_rel(g, o)}"
        assert max_rel(g, u) <= 1e-4, f"output {n} against the unfused plan: {max_rel(g, u)}"


def test_fully_masked_rows_and_large_scores(cuda, oracle, monkeypatch):
    """A mask with empty rows (every score takes the fill value) and scores large enough that
    exp would overflow without the row maximum subtracted."""
    F.use(cuda, "cuda")
    rng = np.random.default_rng(3)
    shape = (2, 2, 128, 32)
    q, k, v, w = (F.tensor((rng.normal(size=shape) * s).astype("float32")) for s in (6.0, 6.0, 1.0, 1.0))
    m = np.tril(np.ones((128, 128), "float32"))
    m[5] = 0.0
    m[77, :40] = 0.0
    mask = F.tensor(m)

    def fn(q, k, v, w):
        return F.value_and_grad(lambda q, k, v: (attention(q, k, v, mask) * w).sum(), argnums=(0, 1, 2))(q, k, v)
    fused, c, leaves = run(fn, (q, k, v, w), True, monkeypatch)
    assert "attention" in ops_of(c)
    cpu = [np_of(x) for x in oracle.run_plan_blob(c.plan_blob(), [triple(t) for t in leaves])]
    for n, (g, o) in enumerate(zip(fused, cpu)):
        assert np.isfinite(g).all()
        assert max_rel(g, o) <= 1e-4, f"output {n}: {max_rel(g, o)}"


def test_gpt_training_step_with_fused_attention(cuda, oracle, monkeypatch):
    """d256-style layers (T = 256, head size 32) in a whole training step: loss and moments
    against the oracle; the attention key bias's gradient is rounding noise (zero in exact
    arithmetic) and its key third is left out."""
    F.use(cuda, "cuda")
    model = F.gpt.GPT(vocab=48, block=256, d=128, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 48, size=4000, dtype="int32"))
    fused, c, leaves = run(F.gpt.make_train_step(model, opt, 2), (state, tokens), True, monkeypatch)
    assert ops_of(c).count("attention") == 2
    cpu = [np_of(x) for x in oracle.run_plan_blob(c.plan_blob(), [triple(t) for t in leaves])]
    n = len(F.tree_leaves(params))
    d = 128
    for i, (g, o) in enumerate(zip(fused, cpu)):
        if g.dtype.kind != "f":
            assert np.array_equal(g, o)
        elif 2 <= i < 2 + 2 * n:  # moments: the gradients
            if g.shape == (3 * d,):
                keep = np.r_[0:d, 2 * d:3 * d]
                assert max_rel(g[keep], o[keep]) <= 1e-4, f"output {i}"
            else:
                assert max_rel(g, o) <= 1e-4, f"output {i}: {max_rel(g, o)}"
    assert max_rel(fused[-1], cpu[-1]) <= 1e-4


def test_packed_form_with_a_general_mask(cuda, oracle, monkeypatch):
    """A GPT attention layer over a mask that is not causal (the kernels pack it into bits; one
    row has every key masked), in the packed form: values and gradients against the oracle; the
    key third of the q/k/v bias gradient is rounding noise and is left out."""
    F.use(cuda, "cuda")
    rng = np.random.default_rng(11)
    b, t, d, heads = 2, 128, 64, 2
    mk = lambda *s: F.tensor((rng.normal(size=s) * 0.3).astype("float32"))
    p = {"qkv": {"w": mk(d, 3 * d), "b": mk(3 * d)}, "out": {"w": mk(d, d), "b": mk(d)}}
    x, w = mk(b, t, d), mk(b, t, d)
    m = (np.random.default_rng(5).random((t, t)) < 0.6).astype("float32")
    np.fill_diagonal(m, 1.0)
    m[3] = 0.0
    mask = F.tensor(m)

    def fn(p, x, w):
        return F.value_and_grad(lambda p, x: (F.gpt.attention(p, x, heads, mask) * w).sum(), argnums=(0, 1))(p, x)
    got, c, leaves = run(fn, (p, x, w), True, monkeypatch)
    steps = [q for q in json.loads(c._n.plan_summary()) if "op" in q]
    assert [q["args"][0] for q in steps if q["op"] == "attention"] == [[b, t, 3, heads, d // heads]]
    cpu = [np_of(y) for y in oracle.run_plan_blob(c.plan_blob(), [triple(l) for l in leaves])]
    for i, (g, o) in enumerate(zip(got, cpu)):
        assert np.isfinite(g).all()
        if g.shape == (3 * d,):
            keep = np.r_[0:d, 2 * d:3 * d]
            assert max_rel(g[keep], o[keep]) <= 1e-4, f"output {i}"
        else:
            assert max_rel(g, o) <= 1e-4, f"output {i}: {max_rel(g, o)}"
