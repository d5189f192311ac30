// Fused attention on the device: the AttnFwd / AttnBwd operations of the device's own graph
// rewrite (graph.h; optimize.cpp fuse_attention). Per batch entry z of Z, with q, k of shape
// (T, d), v of shape (T, dv) and the (T, T) mask:
//   S = q k^T, Z = where(mask, S / c, fill), m = rowmax(Z), E = exp(Z - m), s = rowsum(E),
//   P = E / s, O = P v                                              (forward)
//   D = rowsum(dO * O), dS = P (dO v^T - D) / c where mask != 0 (else 0),
//   dq = dS k, dk = dS^T q, dv = P^T dO                              (backward)
// The (T, T) matrices S, P and dS never leave the chip. Layouts: q, k [Z][T][d], v, dO [Z][T][dv],
// row-major; the forward writes [Z][T][dv + 2] (O, m, s per row), the backward [Z][T][2 d + dv]
// (dq, dk, dv per row). fp32 only.
#pragma once
#include <cuda_runtime.h>

namespace rgc {

struct AttnShape {
  long long batch = 0;  // Z
  int t = 0, d = 0, dv = 0;
  float c = 1.0f, fill = 0.0f;
  // The mask is the causal pattern (mask[i][j] != 0 exactly where j <= i, a constant lower
  // triangle): the tensor-core kernels then compute its bits from the indices.
  bool causal = false;
  // Packed layout (tensor-core shapes only): heads > 0 means q, k and v are the parts of one
  // (B, T, 3, heads, d) tensor (q, k, v point at parts 0, 1, 2; batch entry b * heads + h; row
  // stride 3 heads d), dO is (B, T, heads, d), and the backward writes the gradient of the
  // (B, T, 3, heads, d) tensor instead of the packed (..., T, 3 d) rows.
  int heads = 0;
};

// One-time setup (shared-memory limits of the tensor-core kernels); before any graph capture.
void attention_init();
// Whether the tensor-core kernels take this shape (T 128 or 256, d = dv 32 or 64); other shapes
// run on CUDA cores.
bool attention_tc_supported(const AttnShape& a);
void attention_fwd(float* out, const float* q, const float* k, const float* v, const float* mask, const AttnShape& a, int* error,
                   cudaStream_t s);
// `scratch`: attention_bwd_scratch_bytes(a) bytes of device memory the two backward kernels pass
// the query statistics through (the dq kernel computes them, the dk / dv kernel reads them).
size_t attention_bwd_scratch_bytes(const AttnShape& a);
void attention_bwd(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd, const float* dout,
                   const AttnShape& a, void* scratch, int* error, cudaStream_t s);

}  // namespace rgc
