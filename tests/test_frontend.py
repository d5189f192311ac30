"""The package's front end against rg's: same graphs, same results (CPU, over the oracle module).

rg's own Python front end exists only in the build container, so the equivalence test skips
elsewhere; the PyTorch comparisons need only this package.
"""
import json

import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from conftest import REFERENCE_EXAMPLES


@pytest.fixture
def fe(oracle):
    F.use(oracle, "cpu")
    yield F


def capture_graph(m, compile_fn):
    seen = []
    orig = m.compile

    def spy(g, outs, ex, lvl, dev, opt):
        seen.append((json.loads(g._describe()), list(outs)))
        return orig(g, outs, ex, lvl, dev, opt)
    m.compile = spy
    try:
        c = compile_fn()
    finally:
        m.compile = orig
    return c, seen[-1]


@pytest.mark.reference
def test_gpt_training_step_graph_is_identical_to_rgs_front_end(fe, oracle, rg_reference):
    import sys
    sys.path.insert(0, REFERENCE_EXAMPLES)
    import gpt as ref_gpt
    rg = rg_reference
    cfg = dict(vocab=96, block=16, d=32, heads=4, layers=2)
    toks = np.random.default_rng(0).integers(0, 96, size=5000, dtype="int32")
    m = ref_gpt.GPT(**cfg)
    p = m.init(rg.random.key(0))
    o = rg.optim.adamw(1e-3, weight_decay=0.01)
    st = {"params": p, "opt": o.init(p), "key": rg.random.key(1)}
    rc, (ref_nodes, ref_outs) = capture_graph(oracle, lambda: rg.compile(ref_gpt.make_train_step(m, o, 8), (st, rg.tensor(toks)), validate="basic"))
    m2 = F.gpt.GPT(**cfg)
    p2 = m2.init(F.random.key(0))
    o2 = F.optim.adamw(1e-3, weight_decay=0.01)
    st2 = {"params": p2, "opt": o2.init(p2), "key": F.random.key(1)}
    oc, (our_nodes, our_outs) = capture_graph(oracle, lambda: F.compile(F.gpt.make_train_step(m2, o2, 8), (st2, F.tensor(toks)), validate="basic"))
    assert ref_outs == our_outs
    assert ref_nodes == our_nodes
    for a, b in zip(rg.tree.leaves(p), F.tree_leaves(p2)):
        np.testing.assert_array_equal(np.asarray(a), b.numpy())
    assert rc.report["graph"] == oc.report["graph"]


@pytest.mark.reference
def test_readme_linear_regression_matches_rgs_front_end(fe, oracle, rg_reference):
    rg = rg_reference
    x = np.random.default_rng(0).normal(size=(256, 8)).astype("float32")
    y = x @ np.arange(8, dtype="float32")

    def loss(w, batch):
        return (((batch[0] @ w) - batch[1]) ** 2).mean()

    def ref_step(w, batch):
        value, g = rg.value_and_grad(loss)(w, batch)
        return w - 0.05 * g, value

    def our_step(w, batch):
        value, g = F.value_and_grad(loss)(w, batch)
        return w - 0.05 * g, value
    rc = rg.compile(ref_step, (rg.zeros(8), (x, y)))
    r1 = rg.run(rc, rg.zeros(8), (x, y), steps=500)
    oc = F.compile(our_step, (F.zeros(8), (F.tensor(x), F.tensor(y))))
    r2 = F.run(oc, F.zeros(8), (F.tensor(x), F.tensor(y)), steps=500)
    assert r1.history["aux"] == r2.history["aux"]
    assert r2.history["aux"][-1] < 1e-3


def torch_gpt_loss(torch, p, x, y, heads):
    Fn = torch.nn.functional

    def ln(q, v):
        d = v - v.mean(-1, keepdim=True)
        return d / ((d * d).mean(-1, keepdim=True) + 1e-5).sqrt() * q["scale"] + q["shift"]
    h = p["tok"]["table"][x] + p["pos"]["table"][torch.arange(x.shape[1])]
    mask = torch.tril(torch.ones(x.shape[1], x.shape[1]))
    for b in p["blocks"]:
        n = ln(b["norm1"], h)
        B, T, D = n.shape
        qkv = (n @ b["attn"]["qkv"]["w"] + b["attn"]["qkv"]["b"]).reshape(B, T, 3, heads, D // heads).permute(2, 0, 3, 1, 4)
        s = qkv[0] @ qkv[1].transpose(-1, -2) / (D // heads) ** 0.5
        s = torch.where(mask != 0, s, torch.tensor(-1e9, dtype=s.dtype))
        a = (Fn.softmax(s, -1) @ qkv[2]).transpose(1, 2).reshape(B, T, D)
        h = h + a @ b["attn"]["out"]["w"] + b["attn"]["out"]["b"]
        z = ln(b["norm2"], h) @ b["fc1"]["w"] + b["fc1"]["b"]
        h = h + Fn.gelu(z, approximate="tanh") @ b["fc2"]["w"] + b["fc2"]["b"]
    logits = ln(p["norm"], h) @ p["head"]["w"]
    return Fn.cross_entropy(logits.reshape(-1, logits.shape[-1]), y.reshape(-1))


def test_gpt_loss_and_every_gradient_match_pytorch_f64(fe):
    """rg's test_framework.py:309-356 bar: loss at 1e-11, gradients at rtol 1e-8, in float64."""
    torch = pytest.importorskip("torch")
    model = F.gpt.GPT(vocab=11, block=6, d=8, heads=2, layers=2)
    params = F.tree_map(lambda v: v.cast("float64"), model.init(F.random.key(7)))
    r = np.random.default_rng(5)
    x = r.integers(0, 11, size=(3, 6)).astype("int32")
    y = r.integers(0, 11, size=(3, 6)).astype("int32")
    value, grads = F.value_and_grad(lambda p, x, y: F.nn.cross_entropy(model(p, x), y))(params, F.tensor(x), F.tensor(y))
    tp = F.tree_map(lambda v: torch.tensor(v.numpy(), requires_grad=True), params)
    tv = torch_gpt_loss(torch, tp, torch.tensor(x).long(), torch.tensor(y).long(), 2)
    tv.backward()
    assert float(value) == pytest.approx(tv.item(), rel=1e-11)
    for g, t in zip(F.tree_leaves(grads), F.tree_leaves(tp)):
        np.testing.assert_allclose(g.numpy(), t.grad.numpy(), rtol=1e-8, atol=1e-10)


def test_gpt_memorises_a_pattern(fe, tmp_path):
    """rg's test_framework.py:378-400: loss below 0.05 within 300 steps with the gradient clipped
    at norm 1, then the parameters survive a checkpoint and the sampler continues the pattern."""
    text = "abcdefgh" * 200
    chars = sorted(set(text))
    tokens = F.tensor(np.array([chars.index(c) for c in text], dtype="int32"))
    cfg = dict(vocab=len(chars), block=8, d=32, heads=2, layers=2)
    model = F.gpt.GPT(**cfg)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(3e-3, weight_decay=0.0, max_grad_norm=1.0)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    step = F.compile(F.gpt.make_train_step(model, opt, 16), (state, tokens), validate="standard", device="cpu")
    assert step.report["status"] == "ok", step.report
    r = F.run(step, state, tokens, steps=300)
    assert r.status == "completed"
    assert abs(r.history["aux"][0] - np.log(len(chars))) < 0.3
    assert r.history["aux"][-1] < 0.05
    path = str(tmp_path / "gpt.safetensors")
    F.checkpoint.save(path, r.state["params"], metadata={"config": json.dumps(cfg)})
    loaded, meta = F.checkpoint.load(path, with_metadata=True)
    sampler = F.gpt.compile_sampler(F.gpt.GPT(**json.loads(meta["config"])), loaded, temperature=0.5, device="cpu")
    out = F.gpt.generate(sampler, 8, [chars.index(c) for c in "abc"], 16)
    assert "".join(chars[t] for t in out) == "defghabcdefghabc"


@pytest.mark.reference
def test_run_chunks_and_callbacks_match_rgs_front_end(fe, oracle, rg_reference):
    """Cycled batch lists, an iterator in chunks with a stopping callback, and a run that goes
    non-finite: status, steps, history and final state equal rg's."""
    rg = rg_reference
    rng = np.random.default_rng(8)
    xs = [rng.normal(size=(16, 4)).astype("float32") for _ in range(3)]
    ys = [x @ np.arange(4, dtype="float32") for x in xs]
    results = []
    for lib in (rg, F):
        def step(w, batch, lib=lib):
            value, g = lib.value_and_grad(lambda w: (((batch[0] @ w) - batch[1]) ** 2).mean())(w)
            return w - 0.05 * g, value

        def blow_up(w, lr, lib=lib):
            return w * lr, (w * w).sum()
        batches = [(lib.tensor(x), lib.tensor(y)) for x, y in zip(xs, ys)]
        c = lib.compile(step, (lib.zeros(4), batches[0]), validate="none")
        cycled = lib.run(c, lib.zeros(4), batches, steps=10)
        calls = []
        stopped = lib.run(c, lib.zeros(4), iter(batches * 5), steps=12, every=4, callback=lambda r: calls.append(r.steps) or r.steps < 8)
        bad = lib.compile(blow_up, (lib.ones(2), lib.tensor(1e20)), validate="standard")
        grew = lib.run(bad, lib.ones(2), lib.tensor(1e20), steps=5)
        results.append(dict(cycled=(cycled.status, cycled.steps, cycled.history, np.asarray(cycled.state).tolist()),
                            stopped=(stopped.status, stopped.steps, calls, stopped.history),
                            grew=(grew.status, grew.nonfinite_step, grew.steps)))
    assert results[0] == results[1]
    assert results[1]["stopped"][0] == "stopped_by_callback"
    assert results[1]["grew"][0] == "stopped_nonfinite"
