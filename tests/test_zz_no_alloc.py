"""rgc_sum_noalloc, called through the C ABI.

The entry point serves callers that may not allocate device memory when they need a sum (code
inside an allocator's own callbacks or out-of-memory handler, a host whose memory pool owns the
whole device heap). It keeps its partial sums in a fixed array inside the library instead of a
scratch buffer. These tests check it against the existing path, a compiled plan's full-tensor
Sum run on the CUDA device, on calls in a row that reuse the array's stale contents, and check
that inputs beyond the array's limit are refused.

This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

import rustautograd_b200
from rustautograd_b200 import frontend as F
from helpers import max_rel

MAX_F32 = 1 << 29
MAX_F64 = 1 << 28


def _lib():
    lib = ctypes.CDLL(rustautograd_b200.LIBRARY)
    lib.rgc_sum_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    lib.rgc_sum_noalloc.restype = ctypes.c_int
    lib.rgc_last_error.restype = ctypes.c_char_p
    return lib


def test_sizes_beyond_the_fixed_scratch_are_refused_before_any_launch(product):
    # The size check comes before any CUDA call, so this runs without a GPU; the pointers are
    # never dereferenced.
    lib = _lib()
    fake = ctypes.c_void_p(256)
    for n, dtype in [(MAX_F32 + 1, 0), (MAX_F64 + 1, 1)]:
        assert lib.rgc_sum_noalloc(fake, n, dtype, fake, None) == -1
        assert b"exceed the fixed scratch" in lib.rgc_last_error()
    assert lib.rgc_sum_noalloc(fake, 10, 2, fake, None) == -1
    assert lib.rgc_sum_noalloc(None, 10, 0, fake, None) == -1


@pytest.mark.gpu
def test_two_calls_in_a_row_match_the_plan_path(cuda):
    import torch
    F.use(cuda, "cuda")
    lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream

    def plan_sum(x):
        c = F.compile(lambda a: a.sum(), (F.tensor(x),), validate="none", device="cuda")
        return F.Tensor(c._n.call([F.tensor(x)._t])[0]).numpy()

    def noalloc_sum(x):
        src = torch.from_numpy(x).cuda()
        dst = torch.full((1,), float("nan"), dtype=src.dtype, device="cuda")
        rc = lib.rgc_sum_noalloc(ctypes.c_void_p(src.data_ptr()), x.size, 0 if x.dtype == np.float32 else 1,
                                 ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(stream))
        assert rc == 0, lib.rgc_last_error()
        torch.cuda.synchronize()
        return dst.cpu().numpy()[0]

    rng = np.random.default_rng(7)
    # A large call fills many partials; the smaller call right after it reads back only the
    # partials it wrote itself, with the first call's stale ones still in the array.
    cases = [rng.normal(size=3_000_001).astype("float32"), rng.normal(size=100_003).astype("float32") + 0.5,
             rng.normal(size=1_234_567).astype("float64"), rng.normal(size=4099).astype("float32")]
    for x in cases:
        got, want = noalloc_sum(x), plan_sum(x)
        assert max_rel(got, want) <= 1e-5, (x.size, got, want)
        assert np.asarray(got).tobytes() == np.asarray(want).reshape(()).tobytes(), (x.size, got, want)

    # A refused size leaves the device usable: a buffer of that size exists, so nothing could
    # read out of bounds even if the check were missing.
    big = torch.empty(MAX_F32 + 1, dtype=torch.float32, device="cuda")
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    assert lib.rgc_sum_noalloc(ctypes.c_void_p(big.data_ptr()), MAX_F32 + 1, 0, ctypes.c_void_p(out.data_ptr()),
                               ctypes.c_void_p(stream)) == -1
    del big
    x = rng.normal(size=50_000).astype("float32")
    assert noalloc_sum(x) == plan_sum(x)
