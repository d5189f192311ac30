"""rustautograd_b200: a CUDA (sm_100a) execution device for rg's compiled step plans.

``rustautograd_b200._rg`` is rg's native module interface (Tensor, Graph, Compiled, compile,
available_devices, DiagnosticError) whose plans execute on the GPU through the C ABI of
``include/rgc.h`` (``lib/librgc_b200.so``). ``rustautograd_b200.frontend`` is a Python front end
that traces rg programs onto it. Importing the package never falls back to a CPU engine: without a
usable B200 the ``cuda`` device is simply not offered.
"""
import os

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
LIBRARY = os.path.join(LIB_DIR, "librgc_b200.so")


def load_native():
    """Imports the `_rg` extension; raises ImportError if it has not been built."""
    from . import _rg
    return _rg
