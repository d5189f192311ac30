import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# rg's own checkout (its python/ and examples/ folders), when one is present on this machine: set
# RG_REFERENCE_ROOT to it. Tests that drive rg's Python front end skip when it is unset.
REFERENCE_ROOT = os.environ.get("RG_REFERENCE_ROOT", "")
REFERENCE_PY = os.path.join(REFERENCE_ROOT, "python") if REFERENCE_ROOT else ""
REFERENCE_EXAMPLES = os.path.join(REFERENCE_ROOT, "examples") if REFERENCE_ROOT else ""


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "reference: needs rg's Python front end (only present in the build container)")


def _build():
    from rustautograd_b200 import build_ext
    build_ext.build_oracle()
    build_ext.build_device()
    build_ext.build_module()


@pytest.fixture(scope="session")
def oracle():
    """The CPU oracle module (test infrastructure): rg's `_rg` interface over the restated interpreter."""
    _build()
    path = os.path.join(ROOT, "oracle", "_build")
    if path not in sys.path:
        sys.path.insert(0, path)
    import _rg_oracle
    return _rg_oracle


@pytest.fixture(scope="session")
def product():
    """The product `_rg` module: plans run on the CUDA device through include/rgc.h."""
    _build()
    from rustautograd_b200 import _rg
    return _rg


@pytest.fixture(scope="session")
def cuda(product):
    if not product.cuda_available():
        pytest.fail("a gpu test ran without a usable sm_100 device: the CUDA path must not be skipped silently")
    return product


@pytest.fixture(scope="session")
def rg_reference(oracle):
    """rg's own Python front end, driven over the oracle module (build container only)."""
    if not REFERENCE_PY or not os.path.isdir(REFERENCE_PY):
        pytest.skip("rg's Python front end is not present (set RG_REFERENCE_ROOT to rg's checkout)")
    sys.modules["rg._rg"] = oracle
    if REFERENCE_PY not in sys.path:
        sys.path.insert(0, REFERENCE_PY)
    import rg
    return rg
