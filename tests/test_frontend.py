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
def test_optimiser_options_build_rgs_graphs(fe, oracle, rg_reference):
    """Gradient clipping, a cosine schedule with warmup, SGD with momentum and RMSprop emit the
    same graphs as rg's optim.py."""
    rg = rg_reference
    shapes = [(4, 3), (3,)]
    rng = np.random.default_rng(3)
    arrays = [rng.normal(size=s).astype("float32") for s in shapes]
    cases = [
        (lambda o: o.adamw(o.cosine_decay(1e-2, 100, warmup_steps=10), max_grad_norm=1.0)),
        (lambda o: o.sgd(0.1, momentum=0.9, max_grad_norm=0.5)),
        (lambda o: o.rmsprop(o.cosine_decay(1e-3, 50))),
        (lambda o: o.adam(1e-3)),
    ]
    for make in cases:
        graphs = []
        for lib, tensor in ((rg, rg.tensor), (F, F.tensor)):
            opt = make(lib.optim)
            params = [tensor(a) for a in arrays]
            grads = [tensor(a * 0.5) for a in arrays]
            state = opt.init(params)

            def step(state, p, g, opt=opt):
                return opt.update(g, state, p)
            graphs.append(capture_graph(oracle, lambda: lib.compile(step, (state, params, grads), validate="basic"))[1])
        assert graphs[0] == graphs[1]


@pytest.mark.reference
def test_gpt_with_dropout_builds_rgs_graph(fe, oracle, rg_reference):
    """examples/gpt.py with dropout_rate 0.1: attention-weight, attention-output and MLP dropout."""
    import sys
    sys.path.insert(0, REFERENCE_EXAMPLES)
    import gpt as ref_gpt
    rg = rg_reference
    cfg = dict(vocab=40, block=8, d=16, heads=2, layers=2, dropout_rate=0.1)
    toks = np.random.default_rng(1).integers(0, 40, size=500, dtype="int32")
    graphs = []
    for lib, mod in ((rg, ref_gpt), (F, F.gpt)):
        m = mod.GPT(**cfg)
        p = m.init(lib.random.key(0))
        o = lib.optim.adamw(1e-3)
        st = {"params": p, "opt": o.init(p), "key": lib.random.key(1)}
        graphs.append(capture_graph(oracle, lambda: lib.compile(mod.make_train_step(m, o, 4), (st, lib.tensor(toks)), validate="basic"))[1])
    assert graphs[0] == graphs[1]


@pytest.mark.reference
def test_nn_layers_losses_and_activations_build_rgs_graphs(fe, oracle, rg_reference):
    rg = rg_reference
    rng = np.random.default_rng(4)
    x_np = rng.normal(size=(3, 5)).astype("float32")
    y_np = (rng.random((3, 5)) > 0.5).astype("float32")
    lab_np = np.array([1, 0, 4], dtype="int32")
    graphs, inits = [], []
    for lib in (rg, F):
        nn = lib.nn
        gru = nn.GRUCell(5, 4)
        seq = nn.Sequential(nn.Linear(5, 6), nn.relu, nn.Linear(6, 5))
        params = {"gru": gru.init(lib.random.key(2)), "seq": seq.init(lib.random.key(3))}
        inits.append([np.asarray(nn.xavier_uniform(lib.random.key(5), (4, 6)).numpy()),
                      np.asarray(nn.kaiming_uniform(lib.random.key(6), (4, 6)).numpy())])

        def loss(p, x, y, lab, nn=nn, gru=gru, seq=seq, lib=lib):
            h = lib.zeros((3, 4))
            for _ in range(3):
                h = gru(p["gru"], x, h)
            z = seq(p["seq"], x)
            return (nn.binary_cross_entropy_with_logits(z, y) + nn.l1_loss(nn.sigmoid(z), y) + nn.softplus(z).mean() + nn.silu(z).mean()
                    + (h * h).mean() + (nn.one_hot(lab, 5) * z).sum() + nn.accuracy(z, lab))

        def step(p, x, y, lab, loss=loss, lib=lib):
            return lib.value_and_grad(loss)(p, x, y, lab)
        args = (params, lib.tensor(x_np), lib.tensor(y_np), lib.tensor(lab_np))
        graphs.append(capture_graph(oracle, lambda: lib.compile(step, args, validate="basic"))[1])
    assert graphs[0] == graphs[1]
    for a, b in zip(inits[0], inits[1]):
        np.testing.assert_array_equal(a, b)


@pytest.mark.reference
def test_core_functions_and_transformations_build_rgs_graphs(fe, oracle, rg_reference):
    """abs, sign, square, clip, flip, broadcast_to, matmul, reshape, transpose, expand_dims,
    stack, ones_like, linspace, var/std, grad with aux, jvp, hessian and custom_vjp emit rg's ops."""
    rg = rg_reference
    rng = np.random.default_rng(7)
    a_np = rng.normal(size=(3, 4)).astype("float32")
    b_np = rng.normal(size=(4, 2)).astype("float32")
    graphs = []
    for lib in (rg, F):
        def softsign(x, lib=lib):
            return x / (1.0 + lib.abs(x))
        softsign = lib.custom_vjp(softsign, lambda args, y, ct, lib=lib: (ct / lib.square(1.0 + lib.abs(args[0])),))

        def f(a, b, lib=lib, softsign=softsign):
            z = lib.matmul(lib.clip(a, -0.5, 0.5), b) + lib.sign(a).sum() * lib.ones_like(lib.transpose(b))[0, 0]
            w = lib.stack([lib.flip(a, 0), lib.reshape(a, 3, 4)], axis=1)
            e = lib.expand_dims(lib.broadcast_to(lib.linspace(0.0, 1.0, 4), (3, 4)), -1)
            return (z * z).mean() + (w * e[:, None, :, 0]).std() + softsign(a).var() + a.sin().sum() + b.cos().sum()

        def step(a, b, lib=lib, f=f):
            (value, aux), g = lib.value_and_grad(lambda a, b: (f(a, b), a.sum()), argnums=(0, 1), has_aux=True)(a, b)
            ga = lib.grad(lambda a: f(a, b))(a)
            y, t = lib.jvp(lambda a: f(a, b), (a,), (lib.ones_like(a),))
            h = lib.hessian(lambda v: (v * v * v).sum())(b[:, 0])
            return value, aux, g, ga, y, t, h
        args = (lib.tensor(a_np), lib.tensor(b_np))
        graphs.append(capture_graph(oracle, lambda: lib.compile(step, args, validate="basic"))[1])
    assert graphs[0] == graphs[1]


@pytest.mark.reference
def test_run_chunks_callbacks_and_inspect_match_rgs_front_end(fe, oracle, rg_reference):
    """Cycled batch lists, an iterator in chunks with a stopping callback, and `inspect` of a run
    that went non-finite: status, steps, history and the replayed diagnosis equal rg's."""
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
        report = lib.inspect(grew)
        results.append(dict(cycled=(cycled.status, cycled.steps, cycled.history, cycled.state.numpy().tolist()),
                            stopped=(stopped.status, stopped.steps, calls, stopped.history),
                            grew=(grew.status, grew.nonfinite_step, grew.steps),
                            report=(report["status"], report.get("repro"), [d["code"] for d in report["diagnostics"]]),
                            compiled_report=lib.inspect(c)["graph"]))
    assert results[0] == results[1]
    assert results[1]["stopped"][0] == "stopped_by_callback"
    assert results[1]["grew"][0] == "stopped_nonfinite"
