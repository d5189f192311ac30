"""BASELINE config 3 on the CUDA device: the e-graph search (optimize="search-linear") reorders
sum(A@B@C@D) and sum(x@(U@V)@x^T) and their gradients; the reordered plan on the GPU matches the
oracle running the same plan within 1e-4 (max-norm relative), and it multiplies far less than
the plan as written."""
import json

import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import compile_and_compare, max_rel

pytestmark = pytest.mark.gpu


def _matmul_flops(c):
    total = 0
    for st in json.loads(c._n.plan_summary()):
        if st.get("op") in ("matmul", "matmul_t"):
            a, (ta, tb) = st["args"][0], st["flags"]
            k = (a[-2] if ta else a[-1]) if len(a) >= 2 else a[0]
            total += 2 * int(np.prod(st["shape"])) * k
    return total


def test_config3_chains_reordered_on_the_gpu(oracle, cuda):
    import bench
    F.use(cuda, "cuda")
    w = bench.WORKLOADS["chain-c3"]
    step = w.losses(F)
    args = w.inputs(F)
    state = [F.zeros(a.shape) for a in args]
    gpu, cpu, c = compile_and_compare(oracle, step, (state, args), optimize="search-linear")
    search = c.report["graph"]["optimization"]["search"]
    assert search["accepted"], search
    for k, (g, x) in enumerate(zip(gpu, cpu)):
        assert max_rel(g, x) <= 1e-4, (k, max_rel(g, x))
    plain = F.compile(step, (state, args), validate="none", device="cuda", optimize="standard")
    assert _matmul_flops(c) < 0.2 * _matmul_flops(plain), (_matmul_flops(c), _matmul_flops(plain))
