"""Control flow and sampling on the CUDA device against the CPU oracle running the same plan:
scan (with gradients through it), while_loop, cond, nested control flow, multi-step runs of
plans that contain them, and the GPT sampler step (ArgTopK, Cumsum, Argmax, Concat, RNG).
Integer outputs are compared bit for bit; float outputs of IEEE-only bodies too, and bodies with
transcendental functions at 1e-5 (max-norm relative)."""
import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import assert_bits_equal, assert_parity, np_of, triple

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _frontend(cuda):
    F.use(cuda, "cuda")
    yield


def rnd(*shape, seed=0, scale=1.0, dtype="float32"):
    return F.tensor((np.random.default_rng(seed).normal(size=shape) * scale).astype(dtype))


def test_scan_rnn_value_and_gradients(oracle):
    w, x = rnd(16, 16, seed=1, scale=0.3), rnd(40, 8, 16, seed=2)

    def loss(w, x):
        def body(h, xt):
            h2 = F.tanh(h @ w + xt)
            return h2, h2.sum()
        h, ys = F.scan(body, F.zeros((8, 16)), x)
        return (h * h).sum() + ys.sum()
    assert_parity(oracle, lambda w, x: F.value_and_grad(loss, argnums=(0, 1))(w, x), (w, x), tol=1e-5)


def test_scan_without_xs_and_reverse_order_outputs(oracle):
    a = rnd(5, seed=3)
    fn = lambda a: F.scan(lambda c, _: (c * 0.5 + 1.0, c * c), a, None, length=7)
    assert_parity(oracle, fn, (a,), exact=True)


def test_while_loop_newton_is_bit_exact(oracle):
    def newton(a):
        return F.while_loop(lambda s: (abs(s[0] * s[0] - a) > 1e-6).cast("float32"),
                            lambda s: (0.5 * (s[0] + a / s[0]), s[1] + 1.0), (a, F.tensor(0.0)))
    for v in [2.0, 10.0, 12345.0]:
        assert_parity(oracle, newton, (F.tensor(v),), exact=True)


def test_while_loop_stops_at_its_iteration_limit(oracle):
    fn = lambda x: F.while_loop(lambda s: F.tensor(1.0) + 0.0 * s.sum(), lambda s: s * 1.5, x, max_iterations=13)
    gpu, cpu, _ = assert_parity(oracle, fn, (rnd(4, seed=4),), exact=True)
    assert np.allclose(gpu[0], rnd(4, seed=4).numpy() * 1.5 ** 13, rtol=1e-6)


@pytest.mark.parametrize("p", [1.0, 0.0])
def test_cond_runs_the_chosen_branch(oracle, p):
    x = rnd(30, 7, seed=5)
    fn = lambda p, x: F.cond(p, lambda v: (v * 2.0, v.sum()), lambda v: (v - 1.0, v.max()), x)
    assert_parity(oracle, fn, (F.tensor(p), x), exact=True)


def test_cond_gradient_and_captured_values(oracle):
    x, w = rnd(12, seed=6), rnd(12, seed=7)

    def loss(x, p):
        y = F.cond(p, lambda v: v * w, lambda v: v * v, x)
        return (y * y).sum()
    for p in [1.0, 0.0]:
        assert_parity(oracle, lambda x, p: F.value_and_grad(loss)(x, p), (x, F.tensor(p)), tol=1e-6)


def test_nested_control_flow(oracle):
    xs = rnd(6, 4, seed=8)

    def fn(xs):
        def body(c, x):
            c2 = F.cond((x.sum() > 0.0).cast("float32"), lambda v: v + x, lambda v: v - x, c)
            n = F.while_loop(lambda s: (s < 3.0).cast("float32"), lambda s: s + 1.0, F.tensor(0.0))
            return c2 * 0.5 + n, c2.max()
        return F.scan(body, F.zeros(4), xs)
    assert_parity(oracle, fn, (xs,), exact=True)


def test_run_of_a_plan_with_control_flow_matches_the_oracle(oracle):
    """A multi-step run whose step holds a while loop and a cond: history and final state."""
    data = rnd(32, seed=9)

    def step(s, d):
        s2 = F.while_loop(lambda v: (v.sum() < 100.0).cast("float32"), lambda v: v * 1.1 + 0.5, s, max_iterations=50)
        s3 = F.cond((d.sum() > 0.0).cast("float32"), lambda v: v * 0.25, lambda v: v * 0.5, s2)
        return s3, s3.sum()
    s0 = F.ones(32)
    c = F.compile(step, (s0, data), validate="none", device="cuda")
    r = F.run(c, s0, data, steps=20)
    st, hist, steps, _ = oracle.run_plan_blob_steps(c.plan_blob(), [(0, 0)], [1], [1], [triple(s0), triple(data)], 20)
    assert steps == 20 and r.steps == 20
    np.testing.assert_array_equal(np.array(r.history["aux"]), np.array(hist[0]))
    assert_bits_equal(r.state.numpy(), np_of(st[0]), "state")


def test_selection_ops_for_sampling(oracle):
    x = rnd(6, 50, seed=10)
    fn = lambda x: (F.top_k(x, 7), F.argsort(x), F.sort(x, descending=True), F.cumsum(x), F.argmax(x, 0), F.nn.top_k_logits(x, 5),
                    F.nn.top_p_logits(x, 0.8))
    assert_parity(oracle, fn, (x,), tol=1e-6)


def test_gpt_sampler_generates_the_oracles_tokens(oracle):
    """The sampler step of examples/gpt.py (top-k, top-p, Gumbel-max categorical, context shift)
    run for 24 tokens in one device-resident run: the token ids match the oracle exactly."""
    model = F.gpt.GPT(vocab=40, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    s = F.gpt.compile_sampler(model, params, temperature=0.8, top_k=10, top_p=0.9, device="cuda")
    ids = ([3] * 16 + [5, 9, 1])[-16:]
    state = {"ctx": F.tensor([ids], "int32"), "key": F.random.key(7)}
    r = F.run(s, state, steps=24)
    leaves = F.flatten(state)[0]
    n = len(leaves)
    st, hist, steps, _ = oracle.run_plan_blob_steps(s.plan_blob(), [(k, k) for k in range(n)], [], [n],
                                                     [triple(F.tensor(l)) for l in leaves], 24)
    assert steps == 24
    np.testing.assert_array_equal(np.array(r.history["aux"]), np.array(hist[0]))


def test_device_side_control_flow_in_a_captured_run(oracle):
    """A run's step graph holds while and cond as conditional graph nodes (the condition set by
    a kernel, no host round trip): nested loops, a loop stopped by its iteration limit, and both
    branches taken across steps, against the oracle step for step."""
    data = rnd(16, seed=11)

    def step(s, d):
        def body(v):
            inner = F.while_loop(lambda u: (u.sum() < 40.0).cast("float32"), lambda u: u + 1.0, v * 0.5, max_iterations=7)
            return F.cond((inner.sum() > 30.0).cast("float32"), lambda w: w * 0.9, lambda w: w * 1.1 + 0.3, inner)
        s2 = F.while_loop(lambda v: (v.max() < 25.0).cast("float32"), body, s, max_iterations=9)
        s3 = F.cond((d.sum() > s2.sum() * 0.01).cast("float32"), lambda v: v * 0.25, lambda v: v * 0.75, s2)
        return s3, s3.sum()
    s0 = F.ones(16)
    c = F.compile(step, (s0, data), validate="none", device="cuda")
    r = F.run(c, s0, data, steps=25)
    st, hist, steps, _ = oracle.run_plan_blob_steps(c.plan_blob(), [(0, 0)], [1], [1], [triple(s0), triple(data)], 25)
    assert steps == 25 and r.steps == 25
    np.testing.assert_array_equal(np.array(r.history["aux"]), np.array(hist[0]))
    assert_bits_equal(r.state.numpy(), np_of(st[0]), "state")
