"""validate on the CUDA device: the CUDA-vs-CPU comparison of compile(validate="standard")
(validate.rs:674-705) and the observe=True statistics, computed in the plan on the device.

The product library contains no CPU interpreter; the comparison takes one from the process
(`_set_reference_runner`). Here the test supplies the oracle. A planted mistake is planted in the
oracle's answer, on the CPU."""
import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import max_rel

pytestmark = pytest.mark.gpu


def _small_gpt():
    model = F.gpt.GPT(vocab=40, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 40, size=4000, dtype="int32"))
    return model, opt, state, tokens


def _check(report, name):
    return next(c for c in report["checks"] if c["name"] == name)


@pytest.fixture
def reference(cuda, oracle):
    def run(blob, inputs):
        return oracle.run_plan_blob(blob, inputs)
    cuda._set_reference_runner(run)
    yield run
    cuda._set_reference_runner(None)


def test_device_check_compares_with_the_cpu_interpreter(cuda, reference):
    F.use(cuda, "cuda")
    x = F.tensor(np.random.default_rng(3).normal(size=(64, 33)).astype("float32"))
    c = F.compile(lambda a: (F.tanh(a) * 2.0 + a.sum(axis=0)).sum(axis=1), (x,), validate="standard", device="cuda")
    dc = _check(c.report, "device_equivalence")
    assert dc["status"] == "pass" and dc["detail"]["max_relative_error"] <= 1e-5, dc


def test_device_check_on_the_gpt_training_step(cuda, reference):
    F.use(cuda, "cuda")
    model, opt, state, tokens = _small_gpt()
    c = F.compile(F.gpt.make_train_step(model, opt, 8), (state, tokens), validate="standard", device="cuda")
    dc = _check(c.report, "device_equivalence")
    assert "max_relative_error" in dc["detail"], dc
    assert c.report["status"] in ("ok", "warning")


def test_device_check_reports_a_mismatch_planted_in_the_oracle(cuda, oracle):
    def wrong(blob, inputs):
        out = oracle.run_plan_blob(blob, inputs)
        data, shape, dtype = out[0]
        v = np.frombuffer(data, dtype=dtype).copy()
        v[0] = v[0] * 1.01 + 1.0
        return [(v.tobytes(), shape, dtype)] + list(out[1:])
    cuda._set_reference_runner(wrong)
    try:
        F.use(cuda, "cuda")
        x = F.tensor(np.random.default_rng(4).normal(size=(16, 8)).astype("float32"))
        c = F.compile(lambda a: a * 3.0 + 1.0, (x,), validate="standard", device="cuda")
    finally:
        cuda._set_reference_runner(None)
    codes = [d["code"] for d in c.report["diagnostics"]]
    assert "DEVICE_MISMATCH" in codes, c.report["diagnostics"]


def test_device_check_is_reported_skipped_without_a_cpu_interpreter(cuda):
    F.use(cuda, "cuda")
    x = F.tensor(np.ones((4, 4), "float32"))
    c = F.compile(lambda a: a + 1.0, (x,), validate="standard", device="cuda")
    assert _check(c.report, "device_equivalence")["detail"]["skipped"] == "no_cpu_reference_in_this_process"


def test_observe_statistics_are_computed_on_the_device(cuda, oracle):
    """observe=True: gradient norms, maxima, zero fractions and relative updates are extra plan
    outputs run on the GPU; `run` records them per step, and they track the oracle."""
    F.use(cuda, "cuda")
    model, opt, state, tokens = _small_gpt()
    c = F.compile(F.gpt.make_train_step(model, opt, 8), (state, tokens), validate="none", device="cuda", observe=True)
    r = F.run(c, state, tokens, steps=5)
    assert "grad.global_norm" in r.history and any(k.startswith("update.") for k in r.history)
    assert all(len(v) == 5 for v in r.history.values())
    F.use(oracle, "cpu")
    model, opt, state, tokens = _small_gpt()
    co = F.compile(F.gpt.make_train_step(model, opt, 8), (state, tokens), validate="none", device="cpu", observe=True)
    ro = F.run(co, state, tokens, steps=5)
    for name in ("grad.global_norm", "aux"):
        assert max_rel(np.array(r.history[name]), np.array(ro.history[name])) <= 1e-3, name


def test_standard_validation_scans_for_nonfinite_values_on_the_device(cuda):
    """The finite observer's common case runs as one device pass over the optimised plan with
    per-step flags; a non-finite value falls back to the step-by-step observer, which names the
    root node."""
    F.use(cuda, "cuda")
    model, opt, state, tokens = _small_gpt()
    c = F.compile(F.gpt.make_train_step(model, opt, 8), (state, tokens), validate="standard", device="cuda")
    finite = _check(c.report, "finite")
    assert finite["nonfinite"]["scan"] == "device" and finite["status"] in ("pass", "warn"), finite
    x = F.tensor(np.array([1.0, -1.0, 4.0], "float32"))
    bad = F.compile(lambda a: F.log(a) * 2.0, (x,), validate="standard", device="cuda")
    finite = _check(bad.report, "finite")
    assert finite["nonfinite"]["scan"] == "stepwise" and finite["nonfinite"]["root_nodes"] >= 1, finite
    assert any(d["code"].startswith("NONFINITE") or d["code"].startswith("LOG") or "DOMAIN" in d["code"] for d in bad.report["diagnostics"])
