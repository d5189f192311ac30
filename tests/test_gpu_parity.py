"""CUDA device vs the CPU oracle on the same compiled plan (the plan blob crosses the C ABI).

Tolerances: integer, index and RNG-bit outputs and every plan made of IEEE +,-,*,/ on small
shapes are bit-exact; transcendental functions differ from glibc by a few ulp (CUDA's expf,
tanhf...), so those outputs are compared at 1e-5 relative (max-norm); training-step losses and
gradients at rg's north-star bound of 1e-4 relative (max-norm, rg's device-check metric).
"""
import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import assert_bits_equal, assert_parity, compile_and_compare, max_rel, np_of, triple

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _frontend(cuda):
    F.use(cuda, "cuda")
    yield


def rnd(*shape, seed=0, dtype="float32", scale=1.0):
    return F.tensor((np.random.default_rng(seed).normal(size=shape) * scale).astype(dtype))


UNARY = [
    ("neg", lambda x: -x, True),
    ("abs", lambda x: abs(x), True),
    ("sign", lambda x: F.op("sign", x), True),
    ("floor", lambda x: F.floor(x * 3.0), True),
    ("sqrt", lambda x: F.sqrt(abs(x)), True),
    ("exp", lambda x: F.exp(x), False),
    ("log", lambda x: F.log(abs(x) + 0.5), False),
    ("sin", lambda x: F.op("sin", x), False),
    ("cos", lambda x: F.op("cos", x), False),
    ("tanh", lambda x: F.tanh(x), False),
]


@pytest.mark.parametrize("name,fn,exact", UNARY, ids=[u[0] for u in UNARY])
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_unary(oracle, name, fn, exact, dtype):
    x = rnd(1000, 37, seed=1, dtype=dtype)
    assert_parity(oracle, fn, (x,), tol=1e-5 if dtype == "float32" else 1e-12, exact=exact)


BINARY = [("add", lambda a, b: a + b), ("sub", lambda a, b: a - b), ("mul", lambda a, b: a * b), ("div", lambda a, b: a / b),
          ("max", F.maximum), ("min", F.minimum), ("gt", lambda a, b: a > b), ("ge", lambda a, b: a >= b)]
SHAPES = [((64, 33), (64, 33)), ((), (64, 33)), ((64, 33), ()), ((64, 33), (33,)), ((64, 1), (64, 33)), ((5, 1, 7), (1, 9, 7)), ((2, 3, 4, 5), (3, 1, 5))]


@pytest.mark.parametrize("name,fn", BINARY, ids=[b[0] for b in BINARY])
@pytest.mark.parametrize("sa,sb", SHAPES)
def test_binary_broadcast_is_bit_exact(oracle, name, fn, sa, sb):
    a, b = rnd(*sa, seed=2), rnd(*sb, seed=3)
    assert_parity(oracle, fn, (a, b), exact=True)


@pytest.mark.parametrize("sa,sb", [
    ((8, 4, 64, 64), (8, 4, 64, 1)),    # softmax normalisation: column broadcast
    ((8, 4, 64, 64), (64, 64)),         # mask: row input
    ((16, 6, 10), (16, 1, 10)),         # middle broadcast, inner run 10 (vectors straddle rows)
    ((9, 6), (9, 1)),                   # inner extent 6: vectors cross the broadcast run
    ((3, 5, 2, 4), (5, 1, 1)),          # extents of 1 merged away
    ((2, 3, 4, 5), (3, 1, 5)),
])
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_broadcast_index_paths_are_bit_exact(oracle, sa, sb, dtype):
    a, b = rnd(*sa, seed=31, dtype=dtype), rnd(*sb, seed=32, dtype=dtype)
    fn = lambda a, b: (a / b, (a * b + 1.0) * a, F.maximum(a, b) - b)
    assert_parity(oracle, fn, (a, b), exact=True)


def test_pow_and_ieee_specials(oracle):
    v = np.array([0.0, -0.0, 1.0, -1.0, 2.5, -2.0, np.inf, -np.inf, np.nan, 1e-30, 3e38, -7.0], dtype="float32")
    x = F.tensor(v)
    e = F.tensor(np.array([2.0, 3.0, 0.5, -1.0, 2.0, 3.0, 2.0, 3.0, 1.0, -2.0, 2.0, 2.0], dtype="float32"))
    fns = lambda a, b: (a ** b, F.maximum(a, b), F.minimum(a, b), F.op("sign", a), a / b, F.exp(a), F.tanh(a), F.sqrt(a), F.floor(a))
    gpu, cpu, _ = compile_and_compare(oracle, fns, (x, e))
    for k, (g, w) in enumerate(zip(gpu, cpu)):
        np.testing.assert_array_equal(np.isnan(g), np.isnan(w), err_msg=f"NaN pattern of output {k}")
        m = ~np.isnan(w)
        np.testing.assert_allclose(g[m], w[m], rtol=2e-6, err_msg=f"output {k}")


@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_division_of_every_special_pair_is_bit_exact(oracle, dtype):
    """x / y over all pairs of signed zeros, denormals, infinities, NaN and ordinary values (zero
    numerators take their own path on the device), alone and inside a fused group."""
    tiny = np.finfo(dtype).smallest_subnormal
    v = np.array([0.0, -0.0, 1.0, -1.5, tiny, -tiny, 1e-30, 3e38, np.inf, -np.inf, np.nan, 7.0], dtype=dtype)
    x = F.tensor(np.repeat(v, v.size))
    y = F.tensor(np.tile(v, v.size))
    assert_parity(oracle, lambda a, b: (a / b, (a * 2.0) / (b + 0.0)), (x, y), exact=True)


@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_causal_softmax_division_with_zero_numerators_is_bit_exact(oracle, dtype):
    """The column-broadcast division of a causal softmax, whose upper triangle is zero."""
    t = 64
    e = np.random.default_rng(41).random((4, 3, t, t)).astype(dtype)
    e[..., np.triu_indices(t, 1)[0], np.triu_indices(t, 1)[1]] = 0.0
    e[0, 0, 0, 0] = -0.0
    s = F.tensor(e.sum(-1, keepdims=True))
    assert_parity(oracle, lambda a, b: a / b, (F.tensor(e), s), exact=True)


def test_where_with_broadcast_masks_is_bit_exact(oracle):
    """`where` materialises broadcasts of its smaller operands; the device reads the sources of
    those of constants and inputs directly (a causal mask, fill constants, a column input) and
    keeps the copy for computed ones."""
    t = 32
    x = rnd(4, 3, t, t, seed=51)
    m = F.tril(t)
    col = F.tensor((np.random.default_rng(52).random((4, 3, t, 1)) > 0.5).astype("float32"))
    fn = lambda x, mi, c: (F.where(m, x, -1e9), F.where(m, x * 2.0, 0.0) + x, F.where(mi, x, -1.0) * x, F.where(c, x, 3.0),
                           F.where((mi + 0.5) > 1.0, x, 0.0))
    assert_parity(oracle, fn, (x, F.tril(t), col), exact=True)


def test_fused_chain_matches_and_forms_groups(oracle):
    x, y = rnd(3, 4096, seed=4), rnd(4096, seed=5)
    fn = lambda a, b: F.tanh(a * 0.7978845608 * (a + 0.044715 * a * a * a)) * b + F.exp(-abs(a)) / (1.0 + b * b)
    gpu, cpu, c = assert_parity(oracle, fn, (x, y), tol=1e-5)
    assert c.report["graph"]["fused_groups"] >= 1


def test_where_and_int_arithmetic_wrap(oracle):
    c = F.tensor((np.arange(24).reshape(4, 6) % 3 == 0).astype("float32"))
    a, b = rnd(4, 6, seed=6), rnd(4, 6, seed=7)
    assert_parity(oracle, lambda c, a, b: F.where(c, a, b), (c, a, b), exact=True)
    i = F.tensor(np.array([2147483647, -2147483648, 5, -7, 123456789], dtype="int32"))
    j = F.tensor(np.array([1, -1, 3, 9, 1000], dtype="int32"))
    assert_parity(oracle, lambda p, q: (p + q, p - q, p * q, p > q, p >= q), (i, j), exact=True)


@pytest.mark.parametrize("axes", [None, 0, 1, 2, (0, 1), (1, 2), (0, 2)])
@pytest.mark.parametrize("kind", ["sum", "max", "min"])
def test_reductions(oracle, axes, kind):
    x = rnd(9, 130, 67, seed=8)
    fn = lambda a: getattr(a, kind)(axis=axes, keepdims=False)
    assert_parity(oracle, fn, (x,), tol=1e-5, exact=kind != "sum")


@pytest.mark.parametrize("shape,axis,dtype", [
    ((8192, 37), 0, "float32"),    # 128 partial rows, element staging
    ((5000, 64), 0, "float32"),    # 16-byte staging
    ((4100, 10), 0, "float64"),
    ((64, 70, 9), (0, 1), "float32"),
    ((140001, 8), 0, "float32"),   # 2188 partial rows: the fold stages three 1024-row chunks
    ((70000, 17), 0, "float32"),   # unaligned columns, 4-byte staging, two chunks
    ((140000, 6), 0, "float64"),   # below rg's parallel threshold: one sequential fold per column
])
@pytest.mark.parametrize("kind", ["sum", "max", "min"])
def test_leading_axis_reductions_keep_rgs_order(oracle, shape, axis, dtype, kind):
    # 64-row partials, then the partials in order: the order of plan.rs:1593-1612, so bit-exact.
    x = rnd(*shape, seed=41, dtype=dtype)
    assert_parity(oracle, lambda a: getattr(a, kind)(axis=axis), (x,), exact=True)


@pytest.mark.parametrize("shape", [(300, 256), (77, 68), (5, 3, 2048), (33, 4)])
def test_row_reductions_vector_loads(oracle, shape):
    x = rnd(*shape, seed=42)
    assert_parity(oracle, lambda a: (a.sum(axis=-1), a.max(axis=-1), a.min(axis=-1)), (x,), tol=1e-5)


@pytest.mark.parametrize("length", [4, 8, 63, 64, 65, 127, 128, 200, 256, 1000])
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_row_sums_keep_rgs_eight_lane_order(oracle, length, dtype):
    # Row sums in fast_sum order (plan.rs:1213-1230): lengths around the kernel's 64-element load
    # batches and its 8-element tail.
    x = rnd(300, length, seed=43, dtype=dtype)
    assert_parity(oracle, lambda a: a.sum(axis=-1), (x,), exact=True)


def test_small_full_sum_is_bit_exact(oracle):
    # rg's eight-lane fast_sum order, reproduced on the device for small tensors.
    for n in [1, 7, 8, 9, 256, 1000, 4099]:
        x = rnd(n, seed=n)
        assert_parity(oracle, lambda a: a.sum(), (x,), exact=True)


@pytest.mark.parametrize("perm", [(1, 0), (0, 2, 1), (2, 0, 1), (1, 0, 2), (2, 0, 3, 1)])
def test_transpose(oracle, perm):
    shape = (5, 7, 9, 11)[: len(perm)]
    assert_parity(oracle, lambda a: a.transpose(perm) * 1.0, (rnd(*shape, seed=9),), exact=True)


def test_structural_copies(oracle):
    x = rnd(6, 10, 12, seed=10)
    fn = lambda a: (a[1:5, ::2, 3:], F.op("broadcast_to", a[:, :1, :], shape=[6, 4, 12]), F.concatenate([a, a * 2.0], 1), a[2], a[:, 3, None])
    assert_parity(oracle, fn, (x,), exact=True)


def test_take_and_take_along_with_clamping(oracle):
    table = rnd(11, 8, seed=11)
    idx = F.tensor(np.array([[3, 0, 10], [12, -1, 5]], dtype="int32"))  # out of range clamps
    along = F.tensor(np.array([[1], [0], [7], [2], [9], [3], [5], [4], [6], [0], [1]], dtype="int32"))
    fn = lambda t, i, j: (F.take(t, i, 0), F.take(t, F.tensor(np.array([1, 7], dtype="int32")), 1), F.take_along_axis(t, j))
    assert_parity(oracle, fn, (table, idx, along), exact=True)


def test_scatter_add_gradients_are_bit_exact(oracle):
    # TakeGrad / TakeAlongGrad: every destination adds its contributions in index order from zero.
    table = rnd(17, 64, seed=12)
    idx = F.tensor(np.random.default_rng(13).integers(0, 17, size=(300,), dtype="int32"))
    lab = F.tensor(np.random.default_rng(14).integers(0, 64, size=(17, 3), dtype="int32"))

    def loss(t, i, l):
        e = F.take(t, i, 0)
        return (e * e * F.tensor(np.linspace(0.5, 2.0, 64).astype("float32"))).sum() + F.take_along_axis(t, l).sum()
    fn = lambda t, i, l: F.value_and_grad(loss)(t, i, l)
    assert_parity(oracle, fn, (table, idx, lab), tol=1e-6)
    # The gradient alone (no full-sum of the loss in the way) must be bit-identical.
    g = lambda t, i, l: F.value_and_grad(loss)(t, i, l)[1]
    assert_parity(oracle, g, (table, idx, lab), exact=True)


@pytest.mark.parametrize("table,n_idx,axis,dtype,skew", [
    ((96, 512), (8, 256), 0, "float32", "zipf"),      # many position chunks, 16-byte staging
    ((40, 37), (3000,), 0, "float32", "uniform"),     # row width not a multiple of 4: element staging
    ((50, 70), (5000,), 0, "float64", "zipf"),
    ((7, 33), (2500,), 0, "float64", "uniform"),
    ((3, 20, 48), (1500,), 1, "float32", "zipf"),     # outer extent 3
    ((30, 64), (4000,), 0, "float32", "clamp"),       # out-of-range indices clamp to the ends
])
def test_scatter_add_hit_lists_are_bit_exact(oracle, table, n_idx, axis, dtype, skew):
    rng = np.random.default_rng(21)
    dim = table[axis]
    if skew == "zipf":
        p = (np.arange(dim) + 1.0) ** -1.1
        idx = rng.choice(dim, size=n_idx, p=p / p.sum())
    elif skew == "clamp":
        idx = rng.integers(-5, dim + 5, size=n_idx)
    else:
        idx = rng.integers(0, dim, size=n_idx)
    t = rnd(*table, seed=22, dtype=dtype)
    i = F.tensor(idx.astype("int32"))
    out_shape = table[:axis] + n_idx + table[axis + 1:]
    w = rnd(*out_shape, seed=23, dtype=dtype)
    g = lambda t, i, w: F.value_and_grad(lambda t, i, w: (F.take(t, i, axis) * w).sum())(t, i, w)[1]
    assert_parity(oracle, g, (t, i, w), exact=True)


@pytest.mark.parametrize("sa,sb,kw", [
    ((37, 19), (19, 23), {}),
    ((4, 37, 19), (19, 23), {}),
    ((4, 37, 19), (4, 19, 23), {}),
    ((3, 1, 7, 5), (1, 2, 5, 6), {}),
    ((19,), (19, 23), {}),
    ((37, 19), (19,), {}),
    ((19, 37), (19, 23), {"ta": True}),
    ((37, 19), (23, 19), {"tb": True}),
])
def test_matmul_small_is_bit_exact(oracle, sa, sb, kw):
    a, b = rnd(*sa, seed=15), rnd(*sb, seed=16)

    def fn(x, y):
        if kw.get("ta"):
            x = F.swapaxes(x, -1, -2)
        if kw.get("tb"):
            y = F.swapaxes(y, -1, -2)
        return x @ y
    assert_parity(oracle, fn, (a, b), exact=True)


TC_CASES = [
    # (a shape, b shape, transpose a, transpose b): all above the exact-SIMT size limit.
    ((513, 300), (300, 260), False, False),
    ((300, 513), (300, 260), True, False),
    ((513, 300), (260, 300), False, True),
    ((300, 513), (260, 300), True, True),
    ((32, 128, 64), (32, 64, 128), False, False),   # attention-like batched product
    ((32, 128, 64), (32, 128, 64), False, True),    # q @ k^T
    ((8, 200, 96), (96, 160), False, False),        # batched A with a shared B (one flattened product)
    ((200, 96), (8, 96, 160), False, False),        # shared A with batched B
    ((4, 2, 130, 100), (4, 2, 100, 36), False, False),  # ragged tiles, two batch dims (exact SIMT size)
    ((16, 2, 130, 101), (16, 2, 101, 36), False, False),  # ragged, K not a multiple of 4
    ((515, 301), (301, 259), False, False),         # odd sizes everywhere
    ((301, 515), (259, 301), True, True),
    ((6000, 160), (6000, 260), True, False),        # weight-gradient shape: split K, both operands MN-major
    ((40, 8000), (8000, 72), False, False),         # one output tile, split K
    ((4000, 96), (50, 96), False, True),            # narrow N (64-wide tiles), B K-major
    ((300, 200), (200, 150), False, False),         # B row pitch not a multiple of 4: packed K-major
    ((8, 257, 64), (8, 64, 129), False, False),     # CTA pairs: one row past a pair tile, the odd CTA's B half mostly past N
    ((3, 1000, 72), (3, 72, 100), False, False),    # CTA pairs with 128-wide tiles
    ((8, 257, 96), (8, 96, 259), False, False),     # short K (staged epilogue): ragged rows, N not a multiple of 4
    ((16, 256, 32), (16, 256, 32), False, True),    # short K, q @ k^T at head size 32
    ((9, 128, 130), (9, 128, 120), True, False),    # four K blocks (the staged epilogue's limit), A MN-major
    ((16, 256, 64), (16, 256, 64), False, True),    # batched CTA pairs, B K-major (q @ k^T at T = 256)
    ((520, 4000), (4000, 300), False, False),       # CTA pairs with split K
]


@pytest.mark.parametrize("sa,sb,ta,tb", TC_CASES)
def test_tensor_core_gemm(oracle, sa, sb, ta, tb):
    """3xTF32 tcgen05 products: within 1e-5 (max-norm relative) of rg's fp32 loop."""
    a, b = rnd(*sa, seed=21), rnd(*sb, seed=22)

    def fn(x, y):
        if ta:
            x = F.swapaxes(x, -1, -2)
        if tb:
            y = F.swapaxes(y, -1, -2)
        return x @ y
    assert_parity(oracle, fn, (a, b), tol=1e-5)


def test_matmul_large_within_tolerance(oracle):
    a, b = rnd(512, 384, seed=17), rnd(384, 640, seed=18)
    assert_parity(oracle, lambda x, y: (x @ y, F.swapaxes(x, 0, 1) @ (x @ y)), (a, b), tol=1e-5)


def test_random_streams_are_bit_exact(oracle):
    key = F.tensor(np.array([7, 11], dtype="int32"))
    fn = lambda k: (F.op("key_split", k, n=5), F.op("random_uniform", k, shape=[1000, 3], dtype="float32"),
                    F.op("random_uniform", k, shape=[999], dtype="float64"), F.random.randint(k, (513,), 0, 97))
    assert_parity(oracle, fn, (key,), exact=True)
    gpu, cpu, _ = compile_and_compare(oracle, lambda k: (F.op("random_normal", k, shape=[4096], dtype="float64"),
                                                          F.op("random_normal", k, shape=[4096], dtype="float32")), (key,))
    assert max_rel(gpu[0], cpu[0]) < 1e-14
    assert max_rel(gpu[1], cpu[1]) < 1e-6


def test_casts_saturate_like_rust(oracle):
    v = np.array([0.5, -0.5, 2.9, -2.9, 3e9, -3e9, np.nan, np.inf, -np.inf, 1e20], dtype="float64")
    x = F.tensor(v)
    fn = lambda a: (a.cast("int32"), a.cast("float32"), a.cast("float32").cast("int32"), a.cast("int32").cast("float64"))
    assert_parity(oracle, fn, (x,), exact=True)


def test_selection_ops(oracle):
    x = F.tensor(np.array([[1.0, 3.0, 3.0, -1.0, np.nan, 2.0], [np.nan, 5.0, 1.0, 5.0, 0.0, -2.0], [0.0, -0.0, 0.0, 1.0, 1.0, 1.0]], dtype="float32"))
    fn = lambda a: (F.op("argmax", a), F.op("arg_top_k", a, k=4), F.op("cumsum", a * 1.0, reverse=False), F.op("cumsum", a * 1.0, reverse=True))
    gpu, cpu, _ = compile_and_compare(oracle, fn, (x,))
    for k in range(2):
        assert_bits_equal(gpu[k], cpu[k], f"output {k}")
    for k in range(2, 4):
        np.testing.assert_array_equal(np.isnan(gpu[k]), np.isnan(cpu[k]))


def linear_regression():
    x = np.random.default_rng(0).normal(size=(256, 8)).astype("float32")
    y = x @ np.arange(8, dtype="float32")

    def loss(w, batch):
        return (((batch[0] @ w) - batch[1]) ** 2).mean()

    def step(w, batch):
        value, g = F.value_and_grad(loss)(w, batch)
        return w - 0.05 * g, value
    return step, x, y


def test_linear_regression_run_is_bit_identical_to_the_oracle(oracle):
    """500 steps, history and final weights bit-for-bit equal to rg's CPU."""
    step, x, y = linear_regression()
    w0 = F.zeros(8)
    c = F.compile(step, (w0, (F.tensor(x), F.tensor(y))), validate="basic", device="cuda")
    r = F.run(c, w0, (F.tensor(x), F.tensor(y)), steps=500)
    assert r.status == "completed" and r.steps == 500
    assert r.history["aux"][-1] < 1e-3
    blob = c.plan_blob()
    ins = [triple(F.zeros(8)), triple(F.tensor(x)), triple(F.tensor(y))]
    st, hist, steps, _ = oracle.run_plan_blob_steps(blob, [(0, 0)], [1, 2], [1], ins, 500)
    assert steps == 500
    np.testing.assert_array_equal(np.array(r.history["aux"]), np.array(hist[0]))
    assert_bits_equal(r.state.numpy(), np_of(st[0]), "final weights")


def test_run_stops_at_the_first_nonfinite_step_like_rg(oracle):
    step, x, y = linear_regression()

    def divergent(w, batch):
        value, g = F.value_and_grad(lambda w, b: (((b[0] @ w) - b[1]) ** 2).mean())(w, batch)
        return w - 40.0 * g, value
    w0 = F.zeros(8)
    c = F.compile(divergent, (w0, (F.tensor(x), F.tensor(y))), validate="none", device="cuda")
    r = F.run(c, w0, (F.tensor(x), F.tensor(y)), steps=1000)
    ins = [triple(F.zeros(8)), triple(F.tensor(x)), triple(F.tensor(y))]
    st, hist, steps, _ = oracle.run_plan_blob_steps(c.plan_blob(), [(0, 0)], [1, 2], [1], ins, 1000)
    assert r.status == "stopped_nonfinite"
    assert r.steps == steps and r.nonfinite_step == steps - 1
    np.testing.assert_array_equal(np.array(r.history["aux"]), np.array(hist[0]))
    assert_bits_equal(r.state.numpy(), np_of(st[0]), "state at the stop")


def small_gpt(batch=8, block=16, d=32, heads=4, layers=2, vocab=40, dtype="float32"):
    model = F.gpt.GPT(vocab=vocab, block=block, d=d, heads=heads, layers=layers)
    params = model.init(F.random.key(0))
    if dtype != "float32":
        params = F.tree_map(lambda v: v.cast(dtype), params)
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, vocab, size=4000, dtype="int32"))
    return model, opt, state, tokens


def test_gpt_loss_and_gradients_match_the_oracle(oracle):
    """The north-star bound: fp32 loss and every gradient within 1e-4 relative (max-norm)."""
    model, opt, state, tokens = small_gpt()
    x = F.tensor(np.random.default_rng(1).integers(0, 40, size=(8, 16), dtype="int32"))
    y = F.tensor(np.random.default_rng(2).integers(0, 40, size=(8, 16), dtype="int32"))

    def fn(p, x, y):
        return F.value_and_grad(lambda p, x, y: F.nn.cross_entropy(model(p, x), y))(p, x, y)
    gpu, cpu, c = assert_parity(oracle, fn, (state["params"], x, y), tol=1e-4)
    assert c.report["graph"]["fused_groups"] > 10


def test_gpt_train_step_matches_the_oracle(oracle):
    """One full step (window sampling, forward, backward, AdamW). Loss, key and moments within
    1e-4; parameters within 1e-4 except where Adam's g / (|g| + eps) meets a gradient at the
    rounding-noise level (the attention key bias has a zero gradient in exact arithmetic):
    there the update may differ by at most the 2 * lr a sign flip of that noise moves it."""
    model, opt, state, tokens = small_gpt()
    step = F.gpt.make_train_step(model, opt, 8)
    gpu, cpu, c = compile_and_compare(oracle, step, (state, tokens))
    n = len(F.tree_leaves(state["params"]))
    # Output order: key, count, mu (n), nu (n), params (n), loss.
    for k, (g, w) in enumerate(zip(gpu, cpu)):
        if g.dtype == np.int32:
            assert_bits_equal(g, w, f"output {k}")
        elif 2 + 2 * n <= k < 2 + 3 * n:
            mu = cpu[2 + (k - 2 - 2 * n)]
            noisy = np.abs(mu) <= 1e-5 * max(np.abs(mu).max(), 1e-30)
            assert max_rel(g[~noisy], w[~noisy]) <= 1e-4 if (~noisy).any() else True, f"parameter {k}"
            assert np.all(np.abs(g - w) <= 2 * 1e-3 + 1e-7), f"parameter {k}"
        else:
            assert max_rel(g, w) <= 1e-4, f"output {k}: {max_rel(g, w)}"


def test_gpt_loss_and_gradients_in_float64(oracle):
    model, opt, state, tokens = small_gpt(dtype="float64")
    x = F.tensor(np.random.default_rng(1).integers(0, 40, size=(4, 16), dtype="int32"))

    def fn(p, x):
        return F.value_and_grad(lambda p, x: F.nn.cross_entropy(model(p, x), x))(p, x)
    assert_parity(oracle, fn, (state["params"], x), tol=1e-10)


def test_gpt_training_run_tracks_the_oracle(oracle):
    model, opt, state, tokens = small_gpt()
    step = F.gpt.make_train_step(model, opt, 8)
    c = F.compile(step, (state, tokens), validate="none", device="cuda")
    r = F.run(c, state, tokens, steps=30)
    assert r.status == "completed"
    leaves = F.flatten((state, tokens))[0]
    n_state = len(leaves) - 1
    st, hist, steps, _ = oracle.run_plan_blob_steps(c.plan_blob(), [(k, k) for k in range(n_state)], [n_state], [n_state],
                                                     [triple(F.tensor(l)) for l in leaves], 30)
    assert steps == 30
    # AdamW amplifies ulp differences over many steps; the loss trajectory stays within 1e-4.
    h_gpu, h_cpu = np.array(r.history["aux"]), np.array(hist[0])
    assert np.max(np.abs(h_gpu - h_cpu) / np.abs(h_cpu)) < 1e-4
    assert h_gpu[-1] < h_gpu[0]
