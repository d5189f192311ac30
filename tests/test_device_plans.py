"""Plans as the CUDA device builds them (its fusion configuration and graph rewrites), run on the
CPU oracle through its "cuda-plan" device, against rg's own CPU plan of the same graph.

The device's one rewrite of its own turns a sum of zero-padded blocks that tile an axis (the
gradient of slices along that axis) into a concatenation; every element is the sum's, except
that a -0 block element stays -0 where the sum gives +0, so results are compared with zeros of
either sign equal.
"""
import json

import numpy as np
import pytest

from rustautograd_b200 import frontend as F


@pytest.fixture(autouse=True)
def _frontend(oracle):
    F.use(oracle, "cpu")
    yield


def plan_ops(c):
    return [p.get("op") for p in json.loads(c._n.plan_summary()) if "op" in p]


def run_both(fn, args):
    out = {}
    for dev in ("cpu", "cuda-plan"):
        c = F.compile(fn, args, validate="none", device=dev)
        leaves = [F.tensor(x) for x in F.flatten(args)[0]]
        out[dev] = ([F.Tensor(g).numpy() for g in c._n.call([t._t for t in leaves])], c)
    return out


def assert_same(a, b):
    assert len(a) == len(b)
    for k, (x, y) in enumerate(zip(a, b)):
        assert x.shape == y.shape and x.dtype == y.dtype, k
        assert np.array_equal(x, y, equal_nan=True), f"output {k} differs"


def slice_grad(bounds, axis=0, shape=(6, 5, 4)):
    """Value and gradient of a sum over slices [a, b) of x along `axis`, each with its own weight:
    the gradient is the sum of the slices' padded gradients."""
    x = F.tensor(np.random.default_rng(3).normal(size=shape).astype("float32"))

    def loss(x):
        total = None
        for i, (a, b) in enumerate(bounds):
            idx = [slice(None)] * len(shape)
            idx[axis] = slice(a, b)
            xs = x[tuple(idx)]
            part = (xs * xs).sum() * float(i + 2)
            total = part if total is None else total + part
        return total
    return F.value_and_grad(loss), (x,)


@pytest.mark.parametrize("bounds,axis", [
    ([(0, 2), (2, 4), (4, 6)], 0),        # tiles axis 0, in order
    ([(3, 6), (0, 3)], 0),                # tiles axis 0, blocks in the other order
    ([(0, 1), (1, 5)], 1),                # tiles axis 1
])
def test_padded_gradient_sums_become_concatenations(bounds, axis):
    fn, args = slice_grad(bounds, axis)
    out = run_both(fn, args)
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    assert "concat" in plan_ops(out["cuda-plan"][1])
    assert "pad" not in plan_ops(out["cuda-plan"][1])
    assert "pad" in plan_ops(out["cpu"][1]), "rg's own plan keeps the padded sum"


@pytest.mark.parametrize("bounds,axis", [
    ([(0, 2), (3, 6)], 0),                # a gap: the zeros between the blocks must stay
    ([(0, 4), (2, 6)], 0),                # overlapping blocks add
])
def test_padded_sums_that_do_not_tile_stay_sums(bounds, axis):
    fn, args = slice_grad(bounds, axis)
    out = run_both(fn, args)
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    assert "concat" not in plan_ops(out["cuda-plan"][1])


def test_blocks_padded_along_two_axes_stay_sums():
    x = F.tensor(np.random.default_rng(4).normal(size=(4, 4)).astype("float32"))
    sq = lambda t: (t * t).sum()
    fn = F.value_and_grad(lambda x: sq(x[0:2, 0:2]) * 3.0 + sq(x[2:4, 2:4]) * 5.0 + sq(x[0:2, 2:4]) + sq(x[2:4, 0:2]) * 7.0)
    out = run_both(fn, (x,))
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    assert "concat" not in plan_ops(out["cuda-plan"][1])


def test_gpt_step_plan_concatenates_the_qkv_gradients():
    """The attention layer's q, k, v split: rg's plan pads each gradient to the full (3, B, H, T,
    hd) tensor and adds; the device's plan concatenates them, with every output unchanged."""
    model = F.gpt.GPT(vocab=32, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 32, size=2000, dtype="int32"))
    out = run_both(F.gpt.make_train_step(model, opt, 8), (state, tokens))
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    assert plan_ops(out["cuda-plan"][1]).count("concat") == 2  # one per layer
    assert "pad" not in plan_ops(out["cuda-plan"][1])


def run_steps(fn, state, data, steps, dev):
    c = F.compile(fn, (state, data), validate="none", device=dev)
    return F.run(c, state, data, steps=steps)


def test_linear_regression_history_matches_rgs_plan():
    """500 steps on the device's plan and on rg's, history bit for bit."""
    x = np.random.default_rng(0).normal(size=(256, 8)).astype("float32")
    y = x @ np.arange(8, dtype="float32")

    def step(w, batch):
        value, g = F.value_and_grad(lambda w, b: (((b[0] @ w) - b[1]) ** 2).mean())(w, batch)
        return w - 0.05 * g, value
    data = (F.tensor(x), F.tensor(y))
    a = run_steps(step, F.zeros(8), data, 500, "cpu")
    b = run_steps(step, F.zeros(8), data, 500, "cuda-plan")
    assert list(a.history["aux"]) == list(b.history["aux"])
    assert np.array_equal(a.state.numpy(), b.state.numpy())


def test_adamw_update_matches_rgs_plan():
    """BASELINE config 2 at a reduced size: the fused AdamW update (hoisted step-count chain,
    dependency-level schedule) against rg's unfused plan, three steps, bit for bit."""
    rng = np.random.default_rng(5)
    shapes = [(64, 64), (64,), (16, 64), (64, 16)]
    mk = lambda s: F.tensor((rng.normal(size=s) * 0.02).astype("float32"))
    params = [mk(s) for s in shapes]
    grads = [mk(s) for s in shapes]
    opt = F.optim.adamw(1e-3, 0.9, 0.999, 1e-8, 0.01)
    state = {"params": params, "opt": opt.init(params)}

    def step(state, g):
        p, o = opt.update(g, state["opt"], state["params"])
        return {"params": p, "opt": o}, o["count"]
    a = run_steps(step, state, grads, 3, "cpu")
    b = run_steps(step, state, grads, 3, "cuda-plan")
    la, lb = F.flatten(a.state)[0], F.flatten(b.state)[0]
    assert len(la) == len(lb)
    for k, (u, v) in enumerate(zip(la, lb)):
        assert np.array_equal(u.numpy(), v.numpy()), f"state leaf {k} differs"


def test_matrix_chain_plan_matches_rgs_plan():
    """BASELINE config 3 at a small size with optimize="search-linear": the device's cost model
    may pick another multiplication order, so values agree to rounding (1e-4, max-norm)."""
    rng = np.random.default_rng(6)
    n = 256
    mk = lambda *s: F.tensor(rng.normal(size=s).astype("float32"))
    args = (mk(n, 16), mk(16, n), mk(n, 16), mk(16, n))
    fn = F.value_and_grad(lambda a, b, c, d: (a @ b @ c @ d).sum(), argnums=(0, 1, 2, 3))
    out = {}
    for dev in ("cpu", "cuda-plan"):
        c = F.compile(fn, args, validate="none", device=dev, optimize="search-linear")
        out[dev] = [F.Tensor(g).numpy() for g in c._n.call([t._t for t in args])]
    for k, (u, v) in enumerate(zip(out["cpu"], out["cuda-plan"])):
        scale = max(float(np.abs(u).max()), 1e-30)
        assert float(np.abs(u.astype(np.float64) - v).max()) / scale <= 1e-4, f"output {k}"


def test_device_plans_recompute_forward_values_inside_their_backward_consumers():
    """rg rematerialises values to bound memory; the device recomputes a forward elementwise value
    inside the backward group that reads it when that needs at most one stored full-size source.
    The GELU of the MLP block then writes only its output (one output, where the plan that keeps
    activations writes seven) and its backward group reads the product h and the incoming gradient
    instead of the intermediates. Every output is unchanged bit for bit."""
    model = F.gpt.GPT(vocab=32, block=32, d=64, heads=4, layers=1)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 32, size=2000, dtype="int32"))
    out = run_both(F.gpt.make_train_step(model, opt, 16), (state, tokens))
    assert_same(out["cpu"][0], out["cuda-plan"][0])
    assert out["cuda-plan"][1].report["graph"]["optimization"]["rematerialized"] > 0
    hidden = 16 * 32 * 4 * 64
    gelu = [p for p in json.loads(out["cuda-plan"][1]._n.plan_summary()) if "tanh" in p.get("fused", "") and p.get("n") == hidden]
    assert len(gelu) == 2, "one forward and one backward group"
    forward, backward = gelu
    assert len(forward["out"]) == 1, "the forward group writes only the activation"
    assert len(backward["out"]) == 1
    assert len(backward["fused"].split(",")) > len(forward["fused"].split(",")), "the backward group recomputes the forward chain"
    produced = set(forward["out"])
    assert not produced & set(backward["in"]), "the backward group does not read the forward group's output"


def test_recomputation_reads_stored_values_only():
    """A forward value with two full-size stored sources stays stored (recomputing it would read
    two tensors to save one), and values read by other kinds of steps are never recomputed."""
    rng = np.random.default_rng(9)
    a, b = (F.tensor(rng.normal(size=(64, 64)).astype("float32")) for _ in range(2))

    def loss(a, b):
        u = (a @ b).tanh()          # one stored source: recomputable
        v = (a @ b.T) * (b @ a)     # two stored sources: stays stored
        return (u * u).sum() + (v * v).sum()
    out = run_both(F.value_and_grad(loss, argnums=(0, 1)), (a, b))
    assert_same(out["cpu"][0], out["cuda-plan"][0])


def test_custom_rules_and_control_flow_through_the_device_plan():
    """Every device plan is rebuilt by the device's recomputation rule: a custom gradient rule,
    scan and cond bodies (differentiated) and a while loop (forward only) give rg's results bit
    for bit."""
    rng = np.random.default_rng(0)
    x = F.tensor(rng.normal(size=(64, 32)).astype("float32"))
    w = F.tensor(rng.normal(size=(32, 32)).astype("float32"))
    soft = F.custom_vjp(lambda v: v / (1.0 + F.abs(v)), lambda a, y, ct: (ct / F.square(1.0 + F.abs(a[0])),))

    def with_rule(w, x):
        h = F.nn.gelu(x @ w)
        return (soft(h) * h).sum()

    def with_bodies(w, x):
        def body(c, r):
            c = F.tanh(c @ w + r)
            return c, (c * c).sum()
        c, ys = F.scan(body, F.zeros((32,)), x)
        return ys.sum() + F.cond(c.sum() > 0.0, lambda a: (a * a).sum(), lambda a: a.sum(), c)

    def with_loop(w, x):
        h = F.nn.softmax(x @ w)
        return F.while_loop(lambda s: s[0] < 5.0, lambda s: (s[0] + 1.0, s[1] * 0.5 + h), (F.tensor(0.0), h))[1]
    for fn in (F.value_and_grad(with_rule, argnums=(0, 1)), F.value_and_grad(with_bodies, argnums=(0, 1)), with_loop):
        out = run_both(fn, (w, x))
        assert_same(out["cpu"][0], out["cuda-plan"][0])
