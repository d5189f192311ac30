// fp32-accurate GEMM on the 5th-generation tensor cores (3xTF32 on tcgen05, TMEM accumulators,
// TMA-fed shared-memory pipeline). See gemm_tc.cu.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace rgc {

// One (possibly batched) product C[z] (m x n, row-major) = op(A[z]) @ op(B[z]).
// A is [m, k] (ta = false) or [k, m] (ta = true); B is [k, n] (tb = false) or [n, k] (tb = true);
// batch z's operands start at z * batch_a / z * batch_b elements (0 = shared operand).
struct TcGemm {
  const float* a = nullptr;
  const float* b = nullptr;
  float* c = nullptr;
  long long m = 0, n = 0, k = 0, batch = 1;
  long long batch_a = 0, batch_b = 0;
  bool ta = false, tb = false;
};

// One-time setup (kernel shared-memory limits, the tensor-map encoder); call before any launch
// that may be captured into a CUDA graph.
void tc_gemm_init();
// Whether the tensor-core path takes this product (fp32 only; alignment and shape limits).
bool tc_gemm_supported(const TcGemm& g);
// Scratch bytes the product needs: packed copies of operands whose row pitch TMA cannot read
// (not a multiple of 16 bytes) and split-K partial sums.
size_t tc_gemm_scratch_bytes(const TcGemm& g);
// Kernel launches one product takes.
int tc_gemm_launches(const TcGemm& g);
// Launches the product; `scratch` holds tc_gemm_scratch_bytes bytes; `error` is a device int set
// non-zero if a pipeline wait in the kernel gave up (it then exits without hanging).
void tc_gemm(const TcGemm& g, void* scratch, int* error, cudaStream_t s);

}  // namespace rgc
