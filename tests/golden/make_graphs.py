"""Records the graphs rg's own Python front end builds for BASELINE's workloads, as fixtures that
pin this package's front end (tests/test_graph_fixtures.py) on machines without rg.

Run in a checkout where rg's sources are present:

    RG_REFERENCE_ROOT=<rg checkout> python tests/golden/make_graphs.py

rg's package is loaded read-only from RG_REFERENCE_ROOT/python, over this repository's CPU oracle
module (rg's `_rg` interface), and examples/gpt.py from RG_REFERENCE_ROOT/examples. For each
workload the fixture holds the node list the engine received (op name, attributes, inputs,
shape, dtype; `_rg.Graph._describe`), the output node ids, and a digest of the example inputs'
bytes (so the parameter initialisation is pinned too). Output: tests/golden/graphs.json.gz.
"""
import gzip
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def workloads(lib, gpt_mod, tensor, compile_fn):
    """(name, thunk) pairs; each thunk compiles one workload with front end `lib` (rg's, or this
    package's in test_graph_fixtures.py: both expose these names)."""
    toks = np.random.default_rng(0).integers(0, 96, size=5000, dtype="int32")

    def gpt_step():
        m = gpt_mod.GPT(vocab=96, block=16, d=32, heads=4, layers=2)
        p = m.init(lib.random.key(0))
        o = lib.optim.adamw(1e-3, weight_decay=0.01)
        st = {"params": p, "opt": o.init(p), "key": lib.random.key(1)}
        return compile_fn(gpt_mod.make_train_step(m, o, 8), (st, tensor(toks)))

    def gpt_clipped():
        m = gpt_mod.GPT(vocab=8, block=8, d=16, heads=2, layers=1)
        p = m.init(lib.random.key(0))
        o = lib.optim.adamw(3e-3, weight_decay=0.0, max_grad_norm=1.0)
        st = {"params": p, "opt": o.init(p), "key": lib.random.key(1)}
        return compile_fn(gpt_mod.make_train_step(m, o, 4), (st, tensor(toks % 8)))

    def sampler():
        m = gpt_mod.GPT(vocab=24, block=8, d=16, heads=2, layers=1)
        return gpt_mod.compile_sampler(m, m.init(lib.random.key(3)), temperature=0.7, top_k=5, top_p=0.9)

    def linreg():
        x = np.random.default_rng(0).normal(size=(256, 8)).astype("float32")
        y = x @ np.arange(8, dtype="float32")

        def step(w, batch):
            value, g = lib.value_and_grad(lambda w, b: (((b[0] @ w) - b[1]) ** 2).mean())(w, batch)
            return w - 0.05 * g, value
        return compile_fn(step, (lib.zeros(8), (tensor(x), tensor(y))))

    def adamw():
        rng = np.random.default_rng(0)
        shapes = [(64, 64), (64,), (16, 64), (64, 16)]
        mk = lambda s: tensor((rng.normal(size=s) * 0.02).astype("float32"))
        params, grads, mu = [mk(s) for s in shapes], [mk(s) for s in shapes], [mk(s) for s in shapes]
        nu = [tensor(np.abs(rng.normal(size=s) * 0.02).astype("float32")) for s in shapes]
        o = lib.optim.adamw(1e-3, 0.9, 0.999, 1e-8, 0.01)
        st = {"params": params, "opt": {"count": lib.full((), 0, "float32"), "mu": mu, "nu": nu}}

        def step(state, g):
            p, s = o.update(g, state["opt"], state["params"])
            return {"params": p, "opt": s}, s["count"]
        return compile_fn(step, (st, grads))

    def chain():
        rng = np.random.default_rng(0)
        mk = lambda *s: tensor(rng.normal(size=s).astype("float32"))
        args = [mk(64, 16), mk(16, 64), mk(64, 16), mk(16, 64), mk(32, 64), mk(64, 32), mk(32, 64)]

        def step(grads, a):
            A, B, C, D, x, u, v = a
            l1, g1 = lib.value_and_grad(lambda a, b, c, d: (a @ b @ c @ d).sum(), argnums=(0, 1, 2, 3))(A, B, C, D)
            l2, g2 = lib.value_and_grad(lambda x, u, v: (x @ (u @ v) @ lib.swapaxes(x, 0, 1)).sum(), argnums=(0, 1, 2))(x, u, v)
            return list(g1) + list(g2), l1 + l2
        return compile_fn(step, ([lib.zeros(a.shape) for a in args], args))

    return [("gpt_train_step", gpt_step), ("gpt_train_step_clipped", gpt_clipped), ("gpt_sampler", sampler), ("linreg_c1", linreg),
            ("adamw_c2", adamw), ("matrix_chain_c3", chain)]


def record(module, compile_thunk):
    """(nodes, outputs, input digest) of the graph the engine module receives from one compile."""
    seen = []
    orig = module.compile

    def spy(g, outs, examples, level, device, optimize):
        seen.append((json.loads(g._describe()), list(outs), [bytes(t.tobytes()) for t in examples]))
        return orig(g, outs, examples, level, device, optimize)
    module.compile = spy
    try:
        compile_thunk()
    finally:
        module.compile = orig
    nodes, outs, blobs = seen[-1]
    digest = hashlib.sha256(b"".join(hashlib.sha256(b).digest() for b in blobs)).hexdigest()
    return {"nodes": nodes, "outputs": outs, "inputs_sha256": digest}


def main():
    ref = os.environ.get("RG_REFERENCE_ROOT")
    if not ref:
        raise SystemExit("set RG_REFERENCE_ROOT to rg's checkout")
    sys.path.insert(0, ROOT)
    from rustautograd_b200 import build_ext
    build_ext.build_oracle()
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_build"))
    import _rg_oracle
    sys.modules["rg._rg"] = _rg_oracle
    sys.path.insert(0, os.path.join(ref, "python"))
    sys.path.insert(0, os.path.join(ref, "examples"))
    import rg
    import gpt as rg_gpt
    out = {}
    for name, thunk in workloads(rg, rg_gpt, rg.tensor, lambda fn, ex: rg.compile(fn, ex, validate="basic")):
        out[name] = record(_rg_oracle, thunk)
        print(name, len(out[name]["nodes"]), "nodes")
    with gzip.open(os.path.join(HERE, "graphs.json.gz"), "wt") as f:
        json.dump(out, f, separators=(",", ":"))


if __name__ == "__main__":
    main()
