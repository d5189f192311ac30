// rgc_sum_noalloc: the full-tensor sum without any device allocation.
//
// Some callers cannot allocate device memory at the moment they need a reduction: code running
// inside a custom allocator's own callbacks or out-of-memory handler, a host that has handed
// the whole device heap to its own pool and forbids cudaMalloc behind its back, or a real-time
// loop where cudaMalloc / cudaFree would synchronise the device. The plan path sums a tensor of
// more than 32768 elements in two kernels whose per-chunk partial sums live in the frame's
// scratch arena; this entry point runs the very same two kernels with the partials in a
// fixed array that is part of the library image instead.
//
// Limits and sharing rules:
//  - The array is NOALLOC_SCRATCH_BYTES (256 KiB) on every GPU that loads this library, held
//    until the process exits. One partial per 8192 input elements gives the maximum n:
//    2^29 float32 or 2^28 float64 elements. Larger inputs are rejected before any launch.
//  - Nothing in the array has to start at zero: each call writes every partial before its
//    second kernel reads it, so stale contents of earlier calls are never used.
//  - Every call on a device shares the one array. Two calls that may run at the same time on
//    the GPU (different streams without ordering between them) race on it and can return wrong
//    sums; order them on one stream, or with events.
//  - The first call on each device (more exactly, in each CUDA context that is current when
//    it is called) does set-up: it looks up the array's device address (cudaGetSymbolAddress,
//    with that device current) and its launches load the two kernels. Make that first call
//    before any stream capture is begun. The address is remembered together with the context it
//    was looked up in, so a reset device or primary context is looked up afresh.
//  - Errors are the launches' own return codes; an error that earlier CUDA work of the caller
//    left pending is neither reported nor cleared by this call.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "rgc.h"
#include "kernels.cuh"

namespace rgc {

int set_last_error(int code, const std::string& msg);

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 256 * 1024;
constexpr long long SUM_CHUNK_ELEMENTS = 8192;   // reduce_full_sum's chunk (one partial each)
constexpr long long SUM_SCRATCH_FREE_MAX = 32768; // at or below this the sum needs no partials
constexpr int MAX_DEVICES = 64;

// Device-side storage of the partial sums. In host code this name is only a stand-in for the
// symbol, never a device address: kernels get the address that cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_sum_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
struct ScratchOf {
  void* context = nullptr;  // the CUDA context the address was looked up in
  void* address = nullptr;
};
ScratchOf g_scratch_of[MAX_DEVICES];

// cuCtxGetCurrent through the runtime's driver entry points (no link against libcuda).
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
#pragma GCC diagnostic push
#pragma GCC diagnostic ignored "-Wdeprecated-declarations"
    cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q);
#pragma GCC diagnostic pop
    return (e == cudaSuccess && q == cudaDriverEntryPointSuccess) ? (CtxGetCurrentFn)f : nullptr;
  }();
  return fn;
}

// The array's device address in the current device's current context, looked up once per
// (device, context) pair.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_last_error(RGC_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= MAX_DEVICES) return set_last_error(RGC_ERR_INVALID, "device ordinal out of range");
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return set_last_error(RGC_ERR_CUDA, "cuCtxGetCurrent is not available from the CUDA runtime");
  void* ctx = nullptr;
  if (get(&ctx) != 0) return set_last_error(RGC_ERR_CUDA, "cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchOf& slot = g_scratch_of[dev];
  if (!ctx || !slot.address || slot.context != ctx) {
    // cudaGetSymbolAddress also makes the device's primary context current when no context is
    // yet; the context is read again after it, so the address is filed under the context the
    // launches will use.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sum_scratch);
    if (e != cudaSuccess || !p)
      return set_last_error(RGC_ERR_CUDA, std::string("cudaGetSymbolAddress of the fixed sum scratch: ") + cudaGetErrorString(e));
    if (get(&ctx) != 0 || !ctx) return set_last_error(RGC_ERR_CUDA, "cuCtxGetCurrent: no current CUDA context");
    slot.context = ctx;
    slot.address = p;
  }
  *out = slot.address;
  return RGC_OK;
}

}  // namespace
}  // namespace rgc

extern "C" __attribute__((visibility("default"))) int rgc_sum_noalloc(const void* src, int64_t n, int dtype, void* dst, void* stream) {
  using namespace rgc;
  set_last_error(RGC_OK, "");
  if (dtype != 0 && dtype != 1) return set_last_error(RGC_ERR_INVALID, "rgc_sum_noalloc: dtype must be 0 (float32) or 1 (float64)");
  if (n < 0) return set_last_error(RGC_ERR_INVALID, "rgc_sum_noalloc: negative element count");
  if (!dst || (n > 0 && !src)) return set_last_error(RGC_ERR_INVALID, "rgc_sum_noalloc: null device pointer");
  EType t = dtype == 0 ? EType::F32 : EType::F64;
  const long long max_n = (long long)(NOALLOC_SCRATCH_BYTES / esize(t)) * SUM_CHUNK_ELEMENTS;
  if (n > max_n)
    return set_last_error(RGC_ERR_INVALID, "rgc_sum_noalloc: " + std::to_string(n) + " elements exceed the fixed scratch's limit of " +
                                               std::to_string(max_n) + (dtype == 0 ? " float32" : " float64") + " elements");
  void* scratch = nullptr;
  if (n > SUM_SCRATCH_FREE_MAX) {
    int rc = scratch_address(&scratch);
    if (rc != RGC_OK) return rc;
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = reduce_full_sum(dst, src, t, (long long)n, scratch, s);
  if (e != cudaSuccess) return set_last_error(RGC_ERR_CUDA, std::string("rgc_sum_noalloc launch: ") + cudaGetErrorString(e));
  return RGC_OK;
}
