"""Row chains (on by default, RGC_ROW_CHAINS=0 turns them off) on the CPU: the plan steps the CUDA device computes as one row
kernel, chosen by the same host code the device uses, run by the oracle's "cuda-plan" device the
way the device runs them. Values a chain does not store are filled with NaN there, so a chain
that fails to store a value some later step reads changes the results. Every result is compared
with rg's own plan of the same graph, bit for bit.
"""
import json

import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from test_device_plans import assert_same, plan_ops, run_both


@pytest.fixture(autouse=True)
def _frontend(oracle, monkeypatch):
    monkeypatch.setenv("RGC_ROW_CHAINS", "1")
    F.use(oracle, "cpu")
    yield


def chains(c):
    return json.loads(c._n.row_chains())


def summary(c):
    return json.loads(c._n.plan_summary())


def gpt_step(d=32, heads=4, layers=2, block=16, batch=8):
    model = F.gpt.GPT(vocab=32, block=block, d=d, heads=heads, layers=layers)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 32, size=2000, dtype="int32"))
    return F.gpt.make_train_step(model, opt, batch), (state, tokens)


def test_gpt_step_with_row_chains_matches_rgs_plan():
    fn, args = gpt_step()
    out = run_both(fn, args)
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    found = chains(out["cuda-plan"][1])
    widths = sorted({int(ch["cols"]) for ch in found})
    # Attention rows (T = 16), LayerNorm rows (d = 32), cross-entropy rows (vocab 32).
    assert 16 in widths and 32 in widths, widths
    assert not chains(out["cpu"][1]), "rg's own plans form no chains"


def test_softmax_chain_stores_what_later_steps_read():
    """The attention softmax: masked scores -> row max -> exp -> row sum -> divide. The chain
    stores the exponentials, the row sums and the probabilities, not the masked scores or the
    row maximum."""
    fn, args = gpt_step(layers=1)
    out = run_both(fn, args)
    c = out["cuda-plan"][1]
    ps = summary(c)
    softmax = [ch for ch in chains(c) if int(ch["cols"]) == 16 and "where" in (ps[int(ch["members"][0])].get("fused") or "")]
    assert softmax, [ps[int(ch["members"][0])] for ch in chains(c)]
    ch = softmax[0]
    kinds = [ps[int(m)].get("fused") or ps[int(m)]["op"] for m in ch["members"]]
    assert kinds[:2] == ["div,where", "max"], kinds
    assert ch["store"][0] == [False] and ch["store"][1] == [False], "masked scores and row maximum stay in the chain"
    assert all(flag for flags in ch["store"][2:] for flag in flags), "exponentials, sums and probabilities are stored"


def test_backward_softmax_chain_defers_the_fill_broadcast(monkeypatch):
    """In the greedy-order plan of a d512 layer (compiled, not run; attention unfused, as the
    device fuses this shape by default), the softmax backward reads a broadcast zero through its
    source; the broadcast step, which writes the slot the chain's first member reads dP from,
    runs after the chain."""
    monkeypatch.setenv("RGC_FUSED_ATTENTION", "0")
    fn, args = gpt_step(d=512, heads=8, layers=1, block=256, batch=512)
    c = F.compile(fn, args, validate="none", device="cuda-plan")
    ps = summary(c)
    deferred = [ch for ch in chains(c) if ch["after"]]
    assert deferred
    for ch in deferred:
        for a in ch["after"]:
            assert ps[int(a)]["op"] == "broadcast_to"
            assert int(ch["first"]) < int(a) < int(ch["last"])


def test_layernorm_and_cross_entropy_chains():
    rng = np.random.default_rng(3)
    x = F.tensor(rng.normal(size=(64, 48)).astype("float32"))
    labels = F.tensor(rng.integers(0, 10, size=(64,), dtype="int32"))
    params = {"norm": {"scale": F.ones(48), "shift": F.zeros(48)},
              "head": {"w": F.random.normal(F.random.key(1), (48, 10)) * 0.02, "b": F.zeros(10)}}

    def loss(p, x, y):
        return F.nn.cross_entropy(F.gpt.linear(p["head"], F.gpt.layer_norm(p["norm"], x)), y)
    out = run_both(F.value_and_grad(loss), (params, x, labels))
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    widths = sorted({int(ch["cols"]) for ch in chains(out["cuda-plan"][1])})
    assert 48 in widths and 10 in widths, widths


def test_training_run_history_with_row_chains():
    """A classifier trained for 30 steps through `run` (device-resident loop semantics): every
    loss in the history and the final parameters match rg's plan bit for bit."""
    rng = np.random.default_rng(4)
    x = F.tensor(rng.normal(size=(128, 16)).astype("float32"))
    y = F.tensor(rng.integers(0, 5, size=(128,), dtype="int32"))
    k1, k2 = F.random.split(F.random.key(2))
    params = {"fc1": {"w": F.random.normal(k1, (16, 32)) * 0.02, "b": F.zeros(32)}, "norm": {"scale": F.ones(32), "shift": F.zeros(32)},
              "fc2": {"w": F.random.normal(k2, (32, 5)) * 0.02, "b": F.zeros(5)}}
    opt = F.optim.adamw(1e-2, weight_decay=0.0)
    state = {"params": params, "opt": opt.init(params)}

    def model(p, x):
        return F.gpt.linear(p["fc2"], F.gpt.layer_norm(p["norm"], F.nn.gelu(F.gpt.linear(p["fc1"], x))))

    def step(state, batch):
        value, g = F.value_and_grad(lambda p: F.nn.cross_entropy(model(p, batch[0]), batch[1]))(state["params"])
        p, o = opt.update(g, state["opt"], state["params"])
        return {"params": p, "opt": o}, value
    runs = {}
    for dev in ("cpu", "cuda-plan"):
        c = F.compile(step, (state, (x, y)), validate="none", device=dev)
        runs[dev] = (F.run(c, state, (x, y), steps=30), c)
    assert chains(runs["cuda-plan"][1])
    assert list(runs["cpu"][0].history["aux"]) == list(runs["cuda-plan"][0].history["aux"])
    for u, v in zip(F.flatten(runs["cpu"][0].state)[0], F.flatten(runs["cuda-plan"][0].state)[0]):
        assert np.array_equal(u.numpy(), v.numpy())


def test_reductions_over_other_axes_and_wide_rows_are_left_alone():
    rng = np.random.default_rng(5)
    x = F.tensor(rng.normal(size=(8, 2048)).astype("float32"))
    wide = F.compile(lambda x: F.exp(x - x.max(axis=-1, keepdims=True)).sum(axis=-1), (x,), validate="none", device="cuda-plan")
    assert not chains(wide), "rows longer than a block of shared memory holds"
    y = F.tensor(rng.normal(size=(64, 32)).astype("float32"))
    cols = F.compile(lambda y: F.exp(y - y.max(axis=0, keepdims=True)).sum(axis=0), (y,), validate="none", device="cuda-plan")
    assert not chains(cols), "column reductions are not row chains"


def test_chains_are_on_by_default_and_off_with_the_switch(monkeypatch):
    monkeypatch.delenv("RGC_ROW_CHAINS", raising=False)
    fn, args = gpt_step(layers=1)
    assert chains(F.compile(fn, args, validate="none", device="cuda-plan"))
    monkeypatch.setenv("RGC_ROW_CHAINS", "0")
    c = F.compile(fn, args, validate="none", device="cuda-plan")
    assert not chains(c)
    assert "sum" in plan_ops(c)


def test_chains_inside_a_scan_body():
    """A softmax-and-normalise recurrence under `scan`: the body plan, built with the device's
    configuration, forms its own chains; value and gradients equal rg's plan bit for bit."""
    rng = np.random.default_rng(6)
    xs = F.tensor(rng.normal(size=(5, 12, 16)).astype("float32"))
    w = F.tensor((rng.normal(size=(16, 16)) * 0.3).astype("float32"))

    def loss(w, xs):
        def body(h, x):
            z = h @ w + x
            p = F.nn.softmax(z)
            mu = p.mean(axis=-1, keepdims=True)
            h = (p - mu) / (((p - mu) ** 2).mean(axis=-1, keepdims=True) + 1e-5).sqrt()
            return h, h.sum()
        h, ys = F.scan(body, F.zeros((12, 16)), xs)
        return (h * h).sum() + ys.sum()
    out = run_both(F.value_and_grad(loss), (w, xs))
    assert_same(out["cpu"][0], out["cuda-plan"][0])


def test_step_costs_count_a_chain_once(monkeypatch):
    """With chains, a chain's first step carries its bytes (each outside slot read once, the
    stored values written) and its other steps none, so per-step times and bytes stay paired;
    the step moves fewer algorithmic bytes than without chains."""
    fn, args = gpt_step(layers=1)
    c = F.compile(fn, args, validate="none", device="cuda-plan")
    with_chains = c._n.step_costs()
    found = chains(c)
    assert found
    for ch in found:
        first = int(ch["first"])
        assert with_chains[first][0] == "row_chain" and with_chains[first][2] > 0
        for m in ch["members"][1:]:
            assert with_chains[int(m)] == ("row_chain", 0.0, 0.0)
    monkeypatch.setenv("RGC_ROW_CHAINS", "0")
    without = F.compile(fn, args, validate="none", device="cuda-plan")._n.step_costs()
    assert sum(b for _, _, b in with_chains) < 0.9 * sum(b for _, _, b in without)
    assert sum(f for _, f, _ in with_chains) == sum(f for _, f, _ in without)
