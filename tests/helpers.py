"""Shared test helpers: run the same compiled plan on the CUDA device and on the CPU oracle."""
import numpy as np

from rustautograd_b200 import frontend as F


def np_of(t):
    """numpy array of a front-end Tensor or a (bytes, shape, dtype) triple."""
    if isinstance(t, tuple):
        data, shape, dtype = t
        return np.frombuffer(data, dtype=dtype).reshape(shape).copy()
    return t.numpy()


def triple(t):
    return (t._t.tobytes(), list(t.shape), t.dtype)


def max_rel(got, want):
    """rg's device-check metric (validate.rs:690-697): max |got - want| over max |want|."""
    got = np.atleast_1d(np.asarray(got, dtype=np.float64))
    want = np.atleast_1d(np.asarray(want, dtype=np.float64))
    if got.size == 0:
        return 0.0
    both_nan = np.isnan(got) & np.isnan(want)
    finite = want[np.isfinite(want)]
    scale = max(np.abs(finite).max() if finite.size else 0.0, 1e-30)
    d = np.abs(got - want)
    d[both_nan | (got == want)] = 0.0
    d[np.isnan(d)] = np.inf
    return float(d.max() / scale)


def assert_bits_equal(g, w, what="value"):
    """Bit-identical, except that any two NaNs match (CUDA and x86 produce different NaN payloads)."""
    g, w = np.asarray(g), np.asarray(w)
    assert g.shape == w.shape and g.dtype == w.dtype, (what, g.shape, w.shape, g.dtype, w.dtype)
    if g.dtype.kind == "f":
        ib = np.int64 if g.dtype == np.float64 else np.int32
        same = (g.view(ib) == w.view(ib)) | (np.isnan(g) & np.isnan(w))
    else:
        same = g == w
    if not same.all():
        bad = np.argwhere(~same)
        idx = tuple(bad[0])
        raise AssertionError(f"{what} differs bitwise at {len(bad)} positions, first {bad[:5].tolist()}: {g[idx]!r} vs {w[idx]!r}")


def compile_and_compare(oracle, fn, args, validate="none", optimize="search-linear"):
    """Compiles `fn` for the CUDA device, runs it there and runs the very same plan blob on the
    CPU oracle. Returns (gpu outputs, oracle outputs) as numpy arrays."""
    c = F.compile(fn, args, validate=validate, device="cuda", optimize=optimize)
    leaves = [F.tensor(l) for l in F.flatten(args)[0]]
    gpu = c._n.call([t._t for t in leaves])
    cpu = oracle.run_plan_blob(c.plan_blob(), [triple(t) for t in leaves])
    return [F.Tensor(g).numpy() for g in gpu], [np_of(x) for x in cpu], c


def assert_parity(oracle, fn, args, tol=1e-4, exact=False, **kw):
    gpu, cpu, c = compile_and_compare(oracle, fn, args, **kw)
    assert len(gpu) == len(cpu)
    for k, (g, w) in enumerate(zip(gpu, cpu)):
        assert g.shape == w.shape and g.dtype == w.dtype, (k, g.shape, w.shape, g.dtype, w.dtype)
        if exact or g.dtype == np.int32:
            assert_bits_equal(g, w, f"output {k}")
        else:
            r = max_rel(g, w)
            assert r <= tol, f"output {k}: max relative error {r} > {tol}"
    return gpu, cpu, c
