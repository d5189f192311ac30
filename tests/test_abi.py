"""The C ABI library loads without a GPU and exports exactly what include/rgc.h declares."""
import ctypes
import os
import re
import subprocess

import rustautograd_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    """Entry points declared in include/: the device ABI (rgc.h) and test support (rgc_test.h)."""
    inc = os.path.join(ROOT, "include")
    text = "".join(open(os.path.join(inc, h)).read() for h in sorted(os.listdir(inc)) if h.endswith(".h"))
    return sorted(set(re.findall(r"\b(rgc_[a-z_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol(product):
    lib = ctypes.CDLL(rustautograd_b200.LIBRARY)
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", rustautograd_b200.LIBRARY], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (rgc_[a-z_]+)", out)))
    assert exported == names, (set(exported) ^ set(names))


def test_availability_query_is_safe_and_errors_are_reported(product):
    lib = ctypes.CDLL(rustautograd_b200.LIBRARY)
    lib.rgc_last_error.restype = ctypes.c_char_p
    assert lib.rgc_available() in (0, 1)
    prog = ctypes.c_void_p()
    # A malformed blob is rejected on the host, before any device work.
    bad = (ctypes.c_uint8 * 8)(*b"NOTAPLAN")
    rc = lib.rgc_program_create(bad, 8, -1, ctypes.byref(prog))
    assert rc < 0 and not prog.value
    assert lib.rgc_last_error()
