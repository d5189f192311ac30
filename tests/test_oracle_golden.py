"""The CPU oracle pinned against rg's own known-answer tests (tests/engine.rs of the reference).

Each test restates one engine.rs test through the `_rg` module interface: the expected values
are the ones engine.rs asserts. These pin the restated interpreter, planner, autodiff and run
loop before the oracle is trusted as the parity reference for the CUDA device.
"""
import json

import numpy as np
import pytest


def T(m, shape, values, dtype="float64"):
    arr = np.asarray(values, dtype=dtype).reshape(shape)
    return m.Tensor(arr.tobytes(), list(shape), dtype)


def vals(t):
    return np.frombuffer(t.tobytes(), dtype=t.dtype).tolist()


def sum_all(m, g, x):
    return g.op("sum", [x], {"axes": list(range(len(g.shape(x)))), "keepdims": False})


def test_broadcasting_and_kernels(oracle):  # engine.rs:47-77
    m = oracle
    g = m.Graph()
    a = g.constant(T(m, [2, 3], [1, 2, 3, 4, 5, 6]))
    b = g.constant(T(m, [3], [10, 20, 30]))
    c = g.constant(T(m, [2, 1], [100, 200]))
    s = g.constant(T(m, [], [2.0]))
    ab = g.op("add", [a, b])
    ac = g.op("mul", [a, c])
    sa = g.op("sub", [s, a])
    tr = g.op("transpose", [a], {"perm": [1, 0]})
    sm = g.op("sum", [a], {"axes": [0], "keepdims": False})
    mx = g.op("max", [a], {"axes": [1], "keepdims": True})
    sl = g.op("slice", [a], {"starts": [1, 1], "stops": [2, 3]})
    mm = g.op("matmul", [a, b])
    r = g.eval([ab, ac, sa, tr, sm, mx, sl, mm])
    assert vals(r[0]) == [11, 22, 33, 14, 25, 36]
    assert vals(r[1]) == [100, 200, 300, 800, 1000, 1200]
    assert vals(r[2]) == [1, 0, -1, -2, -3, -4]
    assert r[3].shape == [3, 2] and vals(r[3]) == [1, 4, 2, 5, 3, 6]
    assert vals(r[4]) == [5, 7, 9]
    assert r[5].shape == [2, 1] and vals(r[5]) == [3, 6]
    assert vals(r[6]) == [5, 6]
    assert vals(r[7]) == [140, 320]


def test_pad_through_the_slice_gradient(oracle):  # engine.rs:47-77 `pad` (reached via VJP of slice)
    m = oracle
    g = m.Graph()
    x = g.input([5], "float64")
    sl = g.op("slice", [x], {"starts": [1], "stops": [4]})
    w = g.constant(T(m, [3], [10, 20, 30]))
    y = sum_all(m, g, g.op("mul", [sl, w]))
    (gx,) = g.grad(y, [x])
    c = m.compile(g, [gx], [T(m, [5], [1, 2, 3, 4, 5])], "basic", "cpu", "none")
    assert vals(c.call([T(m, [5], [1, 2, 3, 4, 5])])[0]) == [0, 10, 20, 30, 0]


def test_static_errors_are_structured(oracle):  # engine.rs:79-91
    m = oracle
    g = m.Graph()
    a = g.constant(T(m, [2, 3], [0] * 6))
    b = g.constant(T(m, [2], [0] * 2))
    with pytest.raises(m.DiagnosticError) as e:
        g.op("add", [a, b])
    assert e.value.diagnostic["code"] == "SHAPE_MISMATCH"
    assert e.value.diagnostic["observation"]["lhs_shape"] == [2, 3]
    with pytest.raises(m.DiagnosticError) as e:
        g.op("matmul", [a, a])
    assert e.value.diagnostic["code"] == "SHAPE_MISMATCH"
    f = g.constant(T(m, [2], [0, 0], "float32"))
    with pytest.raises(m.DiagnosticError) as e:
        g.op("add", [b, f])
    assert e.value.diagnostic["code"] == "DTYPE_MISMATCH"
    with pytest.raises(m.DiagnosticError) as e:
        g.grad(a, [a])
    assert e.value.diagnostic["code"] == "GRAD_NON_SCALAR"


def test_take_concat_argmax_and_int_arithmetic(oracle):  # engine.rs:760-785
    m = oracle
    g = m.Graph()
    x = g.constant(T(m, [3, 2], [1, 2, 3, 4, 5, 6]))
    idx = g.constant(T(m, [2, 2], [2, 0, 1, 1], "int32"))
    a0 = g.op("take", [x, idx], {"axis": 0})
    col = g.constant(T(m, [1], [1], "int32"))
    a1 = g.op("take", [x, col], {"axis": 1})
    along = g.constant(T(m, [3, 1], [1, 0, 1], "int32"))
    ta = g.op("take_along", [x, along])
    c = g.op("concat", [x, x], {"axis": 1})
    am = g.op("argmax", [x])
    one = g.constant(T(m, [], [1], "int32"))
    shifted = g.op("add", [col, one])
    r = g.eval([a0, a1, ta, c, am, shifted])
    assert r[0].shape == [2, 2, 2] and vals(r[0]) == [5, 6, 1, 2, 3, 4, 3, 4]
    assert vals(r[1]) == [2, 4, 6]
    assert vals(r[2]) == [2, 3, 6]
    assert vals(r[3]) == [1, 2, 1, 2, 3, 4, 3, 4, 5, 6, 5, 6]
    assert r[4].dtype == "int32" and vals(r[4]) == [1, 1, 1]
    assert r[5].dtype == "int32" and vals(r[5]) == [2]
    with pytest.raises(m.DiagnosticError) as e:
        g.op("exp", [col])
    assert e.value.diagnostic["code"] == "UNSUPPORTED_DTYPE"
    with pytest.raises(m.DiagnosticError) as e:
        g.op("take", [x, x], {"axis": 0})
    assert e.value.diagnostic["code"] == "DTYPE_MISMATCH"


def test_second_order_through_take(oracle):  # engine.rs:828-844
    m = oracle
    g = m.Graph()
    x = g.input([3], "float64")
    i = g.constant(T(m, [4], [0, 2, 2, 1], "int32"))
    tk = g.op("take", [x, i], {"axis": 0})
    p = g.op("pow", [tk, g.constant(T(m, [], [3.0]))])
    y = sum_all(m, g, p)
    (g1,) = g.grad(y, [x])
    (g2,) = g.grad(sum_all(m, g, g1), [x])
    c = m.compile(g, [g2], [T(m, [3], [1, 2, 3])], "none", "cpu", "none")
    assert vals(c.call([T(m, [3], [1, 2, 3])])[0]) == [6, 12, 36]


def test_custom_vjp_rule_replaces_the_body(oracle):  # engine.rs:870-891
    m = oracle
    g = m.Graph()
    x = g.input([2], "float64")
    ph = g.placeholder([2], "float64")
    rule = g.op("mul", [ph, g.constant(T(m, [], [3.0]))])
    c = g.custom(x, ph, [(x, rule)])
    y = sum_all(m, g, g.op("mul", [c, c]))
    (gx,) = g.grad(y, [x])
    x0 = T(m, [2], [1, 2])
    comp = m.compile(g, [y, gx], [x0], "none", "cpu", "standard")
    out = comp.call([x0])
    assert vals(out[0]) == [5] and vals(out[1]) == [6, 12]


def test_out_of_range_index_is_clamped_and_a_hard_error(oracle):  # engine.rs:892-905
    m = oracle
    g = m.Graph()
    x = g.input([3], "float64")
    i = g.constant(T(m, [2], [5, -1], "int32"))
    o = g.op("take", [x, i], {"axis": 0})
    x0 = T(m, [3], [1, 2, 3])
    c = m.compile(g, [o], [x0], "standard", "cpu", "standard")
    assert vals(c.call([x0])[0]) == [3, 1]
    rep = json.loads(c.report_json)
    assert rep["status"] == "validation_failed"
    assert rep["diagnostics"][0]["code"] == "INDEX_OUT_OF_RANGE"
    assert rep["diagnostics"][0]["observation"]["index_max"] == 5.0


def gd_program(m, lr):  # engine.rs:663-680
    g = m.Graph()
    w, x, y = g.input([], "float64"), g.input([], "float64"), g.input([], "float64")
    p = g.op("mul", [w, x])
    e = g.op("sub", [p, y])
    sq = g.op("mul", [e, e])
    loss = g.op("mul", [sq, g.constant(T(m, [], [0.5]))])
    (gr,) = g.grad(loss, [w])
    nw = g.op("sub", [w, g.op("mul", [gr, g.constant(T(m, [], [lr]))])])
    inputs = [T(m, [], [0.0]), T(m, [], [2.0]), T(m, [], [6.0])]
    return m.compile(g, [nw, loss], inputs, "standard", "cpu", "standard")


def test_run_trains_and_stops_on_nonfinite_with_replay(oracle):  # engine.rs:681-702
    m = oracle
    batch = [[T(m, [], [2.0]), T(m, [], [6.0])]]
    c = gd_program(m, 0.1)
    st, outs, hist, steps, bad, secs = c.run([(0, 0)], [1, 2], [1], [T(m, [], [0.0])], batch, 200)
    assert steps == 200 and bad is None
    assert abs(vals(st[0])[0] - 3.0) < 1e-9
    assert hist[0][199] < 1e-15
    assert c.replay([(0, 0)], [1, 2], [1], [T(m, [], [0.0])], batch, 200) is None
    c = gd_program(m, 1000.0)
    st, outs, hist, steps, bad, secs = c.run([(0, 0)], [1, 2], [1], [T(m, [], [0.0])], batch, 10000)
    assert bad is not None and bad < 10000
    k, _, state = c.replay([(0, 0)], [1, 2], [1], [T(m, [], [0.0])], batch, 10000)
    assert k <= bad and state[0].is_finite()
    report = json.loads(c.check([state[0], batch[0][0], batch[0][1]]))
    assert report["status"] == "validation_failed"


def test_run_matches_repeated_calls_exactly_and_cycles_batches(oracle):  # engine.rs:703-717
    m = oracle
    c = gd_program(m, 0.01)
    batches = [[T(m, [], [1.0]), T(m, [], [2.0])], [T(m, [], [3.0]), T(m, [], [1.0])], [T(m, [], [-2.0]), T(m, [], [0.5])]]
    st, outs, hist, steps, bad, secs = c.run([(0, 0)], [1, 2], [1], [T(m, [], [0.5])], batches, 10)
    w = T(m, [], [0.5])
    for k in range(10):
        b = batches[k % 3]
        r = c.call([w, b[0], b[1]])
        assert vals(r[1])[0] == hist[0][k], f"history at step {k}"
        w = r[0]
    assert vals(st[0]) == vals(w)


def test_run_handles_state_passthrough_and_swap(oracle):  # engine.rs:718-730
    m = oracle
    g = m.Graph()
    a, b = g.input([2], "float64"), g.input([2], "float64")
    inputs = [T(m, [2], [1, 2]), T(m, [2], [3, 4])]
    c = m.compile(g, [b, a], inputs, "basic", "cpu", "standard")
    st, *_ = c.run([(0, 0), (1, 1)], [], [], inputs, [], 3)
    assert vals(st[0]) == [3, 4] and vals(st[1]) == [1, 2]


def test_random_streams_are_deterministic_uniform_and_normal(oracle):  # engine.rs:845-869
    m = oracle
    key = T(m, [2], [7, 11], "int32")
    g = m.Graph()
    k = g.input([2], "int32")
    u = g.op("random_uniform", [k], {"shape": [100000], "dtype": "float32"})
    n = g.op("random_normal", [k], {"shape": [100000], "dtype": "float64"})
    ks = g.op("key_split", [k], {"n": 3})
    c = m.compile(g, [u, n, ks], [key], "none", "cpu", "none")
    m.set_threads(1)
    serial = c.call([key])
    m.set_threads(8)
    parallel = c.call([key])
    assert [x.tobytes() for x in serial] == [x.tobytes() for x in parallel], "stream must not depend on threads"
    us, ns = np.array(vals(serial[0])), np.array(vals(serial[1]))
    assert ((us >= 0) & (us < 1)).all()
    assert abs(us.mean() - 0.5) < 0.005 and abs(us.var() - 1 / 12) < 0.002
    assert abs(ns.mean()) < 0.02 and abs(ns.var() - 1) < 0.02
    tail = (np.abs(ns) > 1.96).mean()
    assert abs(tail - 0.05) < 0.003
    split = vals(serial[2])
    assert serial[2].shape == [3, 2] and split[0] != split[2] and split[2] != split[4]
    other = c.call([T(m, [2], [7, 12], "int32")])
    assert other[0].tobytes() != serial[0].tobytes()


def test_parallel_kernels_ignore_thread_count(oracle):  # engine.rs:945-977
    m = oracle
    a, b, cc = 128, 100, 100
    xs = np.sin(np.arange(a * b * cc) * 0.37)
    x0 = T(m, [a, b, cc], xs, "float32")
    g = m.Graph()
    x = g.input([a, b, cc], "float32")
    outs = [g.op("transpose", [x], {"perm": [2, 0, 1]}), g.op("transpose", [x], {"perm": [1, 0, 2]}),
            g.op("max", [x], {"axes": [2], "keepdims": True}), g.op("sum", [x], {"axes": [2], "keepdims": False}),
            g.op("sum", [x], {"axes": [0, 1], "keepdims": True}), g.op("min", [x], {"axes": [0, 1], "keepdims": False})]
    c = m.compile(g, outs, [x0], "none", "cpu", "none")
    res = {}
    for th in (1, 3, 8):
        m.set_threads(th)
        res[th] = [t.tobytes() for t in c.call([x0])]
    m.set_threads(8)
    assert res[1] == res[3] == res[8]
    one = c.call([x0])
    for ci in [0, 7, cc - 1]:
        want = sum(xs[r * cc + ci] for r in range(a * b))
        assert abs(vals(one[4])[ci] - want) < 1e-2
        want_min = float(np.min(np.float32(xs[ci::cc])))
        assert vals(one[5])[ci] == want_min
    assert one[0].shape == [cc, a, b]
    assert vals(one[0])[a * b + 2] == float(np.float32(xs[2 * cc + 1]))


def test_device_switch_reports_unknown_devices(oracle):  # python.rs:268-277
    m = oracle
    g = m.Graph()
    x = g.input([2], "float32")
    with pytest.raises(m.DiagnosticError) as e:
        m.compile(g, [x], [T(m, [2], [1, 2], "float32")], "none", "metal", "standard")
    assert e.value.diagnostic["code"] == "DEVICE_UNAVAILABLE"
    assert e.value.diagnostic["observation"]["available"] == ["cpu"]


# ---- equality saturation (tests/engine.rs:1357-1460) ----

def _eval_graph(m, g, outs, inputs):
    c = m.compile(g, list(outs), inputs, "none", "cpu", "none")
    return [np.frombuffer(t.tobytes(), dtype=t.dtype) for t in c.call(inputs)]


def _chain(m, sizes):
    g = m.Graph()
    ids, inputs = [], []
    for a, b in zip(sizes[:-1], sizes[1:]):
        ids.append(g.input([a, b], "float64"))
        inputs.append(T(m, (a, b), np.sin(np.arange(a * b) * 0.31)))
    v = ids[0]
    for x in ids[1:]:
        v = g.op("matmul", [v, x])
    return g, v, inputs


def _optimal_chain_flops(d):
    n = len(d) - 1
    best = [[0.0] * n for _ in range(n)]
    for length in range(2, n + 1):
        for i in range(n - length + 1):
            j = i + length - 1
            best[i][j] = min(best[i][k] + best[k + 1][j] + d[i] * d[k + 1] * d[j + 1] for k in range(i, j))
    return best[0][n - 1]


def _matmul_flops(g, out):
    nodes = json.loads(g._describe())
    keep, stack = set(), [out]
    while stack:
        i = stack.pop()
        if i not in keep:
            keep.add(i)
            stack.extend(nodes[i]["inputs"])
    total = 0
    for i in keep:
        n = nodes[i]
        if n["op"] == "matmul":
            a, b = nodes[n["inputs"][0]]["shape"], nodes[n["inputs"][1]]["shape"]
            total += int(np.prod(a)) * b[1]
    return total


@pytest.mark.parametrize("sizes", [[30, 35, 15, 5, 10, 20, 25], [1024, 8, 1024, 8, 1024], [4, 300, 2, 500, 3, 200, 6], [10, 20, 30, 40, 30]])
def test_saturation_finds_the_optimal_matrix_chain_order(oracle, sizes):  # engine.rs:1393-1412
    g, out, inputs = _chain(oracle, sizes)
    found = oracle._egraph_search(g, [out], "cpu", 2, 12, 50000)
    h, ids, _ = found if found else (g, [out], None)
    assert _matmul_flops(h, ids[0]) <= _optimal_chain_flops(sizes) * 1.01
    a, b = _eval_graph(oracle, h, ids, inputs)[0], _eval_graph(oracle, g, [out], inputs)[0]
    assert np.max(np.abs(a - b)) <= 1e-9 * max(1.0, np.abs(b).max())


def test_saturation_factors_common_terms_and_rejects_shape_changes(oracle):  # engine.rs:1414-1438
    g = oracle.Graph()
    a, b, c = (g.input([64, 64], "float64") for _ in range(3))
    s = g.op("add", [g.op("matmul", [a, b]), g.op("matmul", [a, c])])
    h, ids, _ = oracle._egraph_search(g, [s], "cpu", 2, 6, 20000)
    assert sum(1 for n in json.loads(h._describe()) if n["op"] == "matmul") == 1
    v = lambda k: T(oracle, (64, 64), np.sin(np.arange(4096) * k * 0.01))
    x, y, z = v(1), v(2), v(3)
    np.testing.assert_allclose(_eval_graph(oracle, h, ids, [x, y, z])[0], _eval_graph(oracle, g, [s], [x, y, z])[0], atol=1e-9)
    # a * (b + c) with broadcasting: factoring [3] and [2, 3] operands must keep the [2, 3] shape.
    g = oracle.Graph()
    a, b, c = g.input([3], "float64"), g.input([3], "float64"), g.input([2, 3], "float64")
    s = g.op("add", [g.op("mul", [a, b]), g.op("mul", [a, c])])
    found = oracle._egraph_search(g, [s], "cpu", 2, 6, 20000)
    h, ids, _ = found if found else (g, [s], None)
    assert json.loads(h._describe())[ids[0]]["shape"] == [2, 3]


def test_exact_rules_never_change_a_bit_on_special_values(oracle):  # engine.rs:1440-1460
    sp = [0.0, -0.0, 1.0, -1.5, 1e300, -1e300, np.inf, -np.inf, np.nan, 1e-300]
    n = len(sp)
    ta = T(oracle, (n * n,), np.repeat(sp, n))
    tb = T(oracle, (n * n,), np.tile(sp, n))
    g = oracle.Graph()
    x, y = g.input([n * n], "float64"), g.input([n * n], "float64")
    nx = g.op("neg", [x])
    outs = [g.op("sub", [g.op("neg", [nx]), y]), g.op("mul", [nx, y]), g.op("div", [nx, y]), g.op("add", [y, x])]
    h, ids, _ = oracle._egraph_search(g, outs, "cpu", 0, 6, 20000)
    want, got = _eval_graph(oracle, g, outs, [ta, tb]), _eval_graph(oracle, h, ids, [ta, tb])
    for u, v in zip(want, got):
        same = (u.view(np.int64) == v.view(np.int64)) | (np.isnan(u) & np.isnan(v))
        assert same.all()


def test_search_linear_reorders_the_config3_chains(oracle):
    """BASELINE config 3 at a quarter scale: `optimize="search-linear"` reorders A@B@C@D and
    x@(U@V)@x^T (forward and gradients) to far fewer multiplications, and the values stay within
    1e-4 of the plan as written."""
    from rustautograd_b200 import frontend as F
    F.use(oracle, "cpu")
    rng = np.random.default_rng(0)
    n = 1024
    mk = lambda *s: F.tensor(rng.normal(size=s).astype("float32"))
    A, B, C, D = mk(n, 16), mk(16, n), mk(n, 16), mk(16, n)
    x, U, V = mk(256, n), mk(n, 32), mk(32, n)
    cases = [(lambda a, b, c, d: (a @ b @ c @ d).sum(), (A, B, C, D)), (lambda x, u, v: (x @ (u @ v) @ F.swapaxes(x, 0, 1)).sum(), (x, U, V))]
    for fn, args in cases:
        g = lambda *a: F.value_and_grad(fn, argnums=tuple(range(len(a))))(*a)
        opt = F.compile(g, args, validate="none", device="cpu", optimize="search-linear")
        std = F.compile(g, args, validate="none", device="cpu", optimize="standard")
        search = opt.report["graph"]["optimization"]["search"]
        assert search["accepted"] and search["cost_after"] < 0.5 * search["cost_before"], search
        for u, w in zip(F.tree_leaves(opt(*args)), F.tree_leaves(std(*args))):
            u, w = np.asarray(u.numpy(), np.float64), np.asarray(w.numpy(), np.float64)
            assert np.abs(u - w).max() <= 1e-4 * np.abs(w).max()
