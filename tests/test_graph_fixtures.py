"""This package's front end records the graphs rg's own front end records, for BASELINE's
workloads: the GPT training step (configs 4 and 5, also with gradient clipping), the GPT sampler,
the linear regression (config 1), AdamW (config 2) and the matrix chains (config 3).

The fixtures (tests/golden/graphs.json.gz) were recorded from rg's python/rg and examples/gpt.py
by tests/golden/make_graphs.py; this test needs neither. Equal node lists (op, attributes,
inputs, shape, dtype) and equal example-input bytes mean the engine compiles the same plan from
the same parameters.
"""
import gzip
import json
import os
import sys

import pytest

from rustautograd_b200 import frontend as F

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_graphs  # noqa: E402

FIXTURES = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "graphs.json.gz")


@pytest.fixture(scope="module")
def recorded():
    with gzip.open(FIXTURES, "rt") as f:
        return json.load(f)


@pytest.mark.parametrize("name", ["gpt_train_step", "gpt_train_step_clipped", "gpt_sampler", "linreg_c1", "adamw_c2", "matrix_chain_c3"])
def test_front_end_records_rgs_graph(oracle, recorded, name):
    F.use(oracle, "cpu")
    thunk = dict(make_graphs.workloads(F, F.gpt, F.tensor, lambda fn, ex: F.compile(fn, ex, validate="basic")))[name]
    ours = make_graphs.record(oracle, thunk)
    want = recorded[name]
    assert len(ours["nodes"]) == len(want["nodes"])
    for k, (a, b) in enumerate(zip(ours["nodes"], want["nodes"])):
        assert a == b, f"node {k}: {a} != {b}"
    assert ours["outputs"] == want["outputs"]
    assert ours["inputs_sha256"] == want["inputs_sha256"], "example inputs (parameter initialisation) differ"
