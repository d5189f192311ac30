// Fused attention (attention.cuh) on sm_100a.
//
// Tensor-core path (T = 128 or 256, d = dv = 32 or 64): 3xTF32 products on tcgen05 with fp32
// accumulators in TMEM, as in gemm_tc.cu (hi = the raw fp32 value, which the tensor core reads as
// TF32; lo = x - trunc_tf32(x); A B = A_hi B_hi + A_hi B_lo + A_lo B_hi). Operand tiles are staged
// in shared memory by the CTA's own threads, which write hi and lo in the K-major 128-byte-swizzle
// layout the MMA descriptors read (a transposed operand is written transposed, so every operand is
// K-major). One CTA of four warps takes 128 query rows of one batch entry; thread i owns row i
// (TMEM lane i), so row statistics need no exchange:
//   forward   S = q k^T into TMEM (T columns); two passes over S give each row's max and exp-sum
//             (the sum in key order); then per 32-key chunk P = exp(Z - m) / s goes to shared
//             memory (hi and lo, double-buffered) and O += P v accumulates in TMEM.
//   backward  two kernels, each recomputing the scores: k_attn_dq_tc (one thread per query row)
//             forms dS chunk by chunk and accumulates dq = dS k; k_attn_dkdv_tc (one thread per
//             key row) works on the transposes, forming P^T and dS^T and accumulating
//             dv = P^T dO and dk = dS^T q. D = rowsum(dO * O) comes from the forward's O.
//
// CUDA-core path (any other T up to 1024 and any d): one warp per row, for the small shapes of
// tests and models outside the tensor-core tiles.
//
// Every mbarrier wait is bounded (tc_common.cuh); on expiry the kernel records an error code,
// waits (bounded) for the products it issued, frees its TMEM and returns.
#include "attention.cuh"

#include <cmath>
#include <mutex>
#include <stdexcept>
#include <string>

#include "tc_common.cuh"

namespace rgc {

namespace {

using namespace tc;

constexpr unsigned FULL = 0xffffffffu;

// ---------------------------------------------------------------------------------------------
// CUDA-core kernels
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ float nan_max(float m, float z) { return (z > m || z != z) ? z : m; }

// One warp per query row (global row z * T + r); per-warp scratch of T floats.
__global__ void k_attn_fwd_simt(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                const float* __restrict__ mask, long long rows, int T, int D, int DV, float c, float fill) {
  extern __shared__ float zs[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 4 + warp;
  if (row >= rows) return;
  const long long z = row / T;
  const int r = (int)(row - z * T);
  const float* qr = q + row * D;
  const float* kz = k + z * T * D;
  const float* vz = v + z * T * DV;
  float* zr = zs + warp * T;
  float m = -INFINITY;
  for (int j = lane; j < T; j += 32) {
    float acc = 0.0f;
    for (int e = 0; e < D; ++e) acc = acc + qr[e] * kz[(long long)j * D + e];
    const float zz = mask[(long long)r * T + j] != 0.0f ? acc / c : fill;
    zr[j] = zz;
    m = nan_max(m, zz);
  }
  for (int o = 16; o; o >>= 1) m = nan_max(m, __shfl_xor_sync(FULL, m, o));
  __syncwarp();
  float sum = 0.0f;
  for (int j = lane; j < T; j += 32) {
    const float e = expf(zr[j] - m);
    zr[j] = e;
    sum = sum + e;
  }
  for (int o = 16; o; o >>= 1) sum = sum + __shfl_xor_sync(FULL, sum, o);
  __syncwarp();
  float* orow = out + row * (DV + 2);
  for (int e = lane; e < DV; e += 32) {
    float acc = 0.0f;
    for (int j = 0; j < T; ++j) acc = acc + (zr[j] / sum) * vz[(long long)j * DV + e];
    orow[e] = acc;
  }
  if (lane == 0) {
    orow[DV] = m;
    orow[DV + 1] = sum;
  }
}

// dq: one warp per query row.
__global__ void k_attn_dq_simt(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               const float* __restrict__ mask, const float* __restrict__ fwd, const float* __restrict__ dout, long long rows, int T,
                               int D, int DV, float c, float fill) {
  extern __shared__ float dss[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 4 + warp;
  if (row >= rows) return;
  const long long z = row / T;
  const int r = (int)(row - z * T);
  const float* qr = q + row * D;
  const float* kz = k + z * T * D;
  const float* vz = v + z * T * DV;
  const float* fw = fwd + row * (DV + 2);
  const float* dor = dout + row * DV;
  const float m = fw[DV], sum = fw[DV + 1];
  float Dr = 0.0f;
  for (int e = lane; e < DV; e += 32) Dr = Dr + dor[e] * fw[e];
  for (int o = 16; o; o >>= 1) Dr = Dr + __shfl_xor_sync(FULL, Dr, o);
  float* ds = dss + warp * T;
  for (int j = lane; j < T; j += 32) {
    float acc = 0.0f;
    for (int e = 0; e < D; ++e) acc = acc + qr[e] * kz[(long long)j * D + e];
    const bool on = mask[(long long)r * T + j] != 0.0f;
    const float p = expf((on ? acc / c : fill) - m) / sum;
    float dp = 0.0f;
    for (int e = 0; e < DV; ++e) dp = dp + dor[e] * vz[(long long)j * DV + e];
    ds[j] = on ? p * (dp - Dr) / c : 0.0f;
  }
  __syncwarp();
  float* g = out + row * (2 * D + DV);
  for (int e = lane; e < D; e += 32) {
    float acc = 0.0f;
    for (int j = 0; j < T; ++j) acc = acc + ds[j] * kz[(long long)j * D + e];
    g[e] = acc;
  }
}

// dk and dv: one warp per key row j.
__global__ void k_attn_dkdv_simt(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                 const float* __restrict__ mask, const float* __restrict__ fwd, const float* __restrict__ dout, long long rows,
                                 int T, int D, int DV, float c, float fill) {
  extern __shared__ float sh[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 4 + warp;
  if (row >= rows) return;
  const long long z = row / T;
  const int j = (int)(row - z * T);
  const float* qz = q + z * T * D;
  const float* kj = k + row * D;
  const float* vj = v + row * DV;
  const float* fz = fwd + z * T * (DV + 2);
  const float* dz = dout + z * T * DV;
  float* P = sh + warp * 2 * T;
  float* DS = P + T;
  for (int r = lane; r < T; r += 32) {
    const float* fw = fz + (long long)r * (DV + 2);
    const float* dor = dz + (long long)r * DV;
    float Dr = 0.0f, dp = 0.0f, acc = 0.0f;
    for (int e = 0; e < DV; ++e) {
      Dr = Dr + dor[e] * fw[e];
      dp = dp + dor[e] * vj[e];
    }
    for (int e = 0; e < D; ++e) acc = acc + qz[(long long)r * D + e] * kj[e];
    const bool on = mask[(long long)r * T + j] != 0.0f;
    const float p = expf((on ? acc / c : fill) - fw[DV]) / fw[DV + 1];
    P[r] = p;
    DS[r] = on ? p * (dp - Dr) / c : 0.0f;
  }
  __syncwarp();
  float* g = out + row * (2 * D + DV);
  for (int e = lane; e < D; e += 32) {
    float acc = 0.0f;
    for (int r = 0; r < T; ++r) acc = acc + DS[r] * qz[(long long)r * D + e];
    g[D + e] = acc;
  }
  for (int e = lane; e < DV; e += 32) {
    float acc = 0.0f;
    for (int r = 0; r < T; ++r) acc = acc + P[r] * dz[(long long)r * DV + e];
    g[2 * D + e] = acc;
  }
}

// ---------------------------------------------------------------------------------------------
// Tensor-core building blocks
// ---------------------------------------------------------------------------------------------

constexpr int TC_THREADS = 128;

// Byte offset of element (row, k) in a K-major tile of R rows whose K extent is cut into 32-wide
// blocks (R x 128 bytes each): 8-row groups of 1024 bytes, 128 bytes per row, and the row's
// 16-byte chunk (k % 32) / 4 stored at chunk position ((k % 32) / 4) ^ (row % 8) — the 128-byte
// swizzle that desc_k describes (the layout TMA's SWIZZLE_128B writes for gemm_tc.cu).
__device__ __forceinline__ uint32_t kmaj(int R, int row, int k) {
  return (uint32_t)((k >> 5) * R * 128 + (row >> 3) * 1024 + (row & 7) * 128 + ((((k & 31) >> 2) ^ (row & 7)) << 4) + ((k & 3) << 2));
}

__device__ __forceinline__ float tf32_lo(float x) { return x - tf32_trunc(x); }

// Rows [0, R) x columns [0, K) of a row-major global block (row stride `ld` floats, 16-byte
// aligned rows) into K-major hi / lo tiles.
__device__ __forceinline__ void stage(uint8_t* hi, uint8_t* lo, const float* src, int R, int K, long long ld) {
  const int k4 = K >> 2;
  for (int i = threadIdx.x; i < R * k4; i += TC_THREADS) {
    const int row = i / k4, col = (i - row * k4) << 2;
    const float4 x = *(const float4*)(src + row * ld + col);
    const uint32_t off = kmaj(R, row, col);
    *(float4*)(hi + off) = x;
    *(float4*)(lo + off) = make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w));
  }
}

// The transpose of a row-major global block: source rows [0, Rs) become the tile's K index and
// source columns [0, Cs) its rows (a K-major tile of Cs rows over K = Rs).
__device__ __forceinline__ void stage_t(uint8_t* hi, uint8_t* lo, const float* src, int Rs, int Cs, long long ld) {
  const int c4 = Cs >> 2;
  for (int i = threadIdx.x; i < Rs * c4; i += TC_THREADS) {
    const int j = i / c4, col = (i - j * c4) << 2;
    const float4 x = *(const float4*)(src + j * ld + col);
    const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t off = kmaj(Cs, col + q, j);
      *(float*)(hi + off) = xs[q];
      *(float*)(lo + off) = tf32_lo(xs[q]);
    }
  }
}

// Instruction descriptor: M x N, TF32 x TF32 -> F32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (128 x N) (+)= A (128 x K) B (N x K)^T in 3xTF32, A and B K-major hi/lo tiles (shared-memory
// addresses; B's tile has N rows). Issued by one thread.
__device__ __forceinline__ void mma3(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl, int N, int K, uint32_t idesc, bool accumulate) {
  for (int kb = 0; kb < K / 32; ++kb) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t ao = (uint32_t)(kb * 128 * 128 + kk * 32), bo = (uint32_t)(kb * N * 128 + kk * 32);
      mma_tf32(d, desc_k(ah + ao), desc_k(bh + bo), idesc, (accumulate || kb || kk) ? 1u : 0u);
      mma_tf32(d, desc_k(ah + ao), desc_k(bl + bo), idesc, 1u);
      mma_tf32(d, desc_k(al + ao), desc_k(bh + bo), idesc, 1u);
    }
  }
}

__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int T, int D> struct FwdLayout {
  static constexpr int QB = 128 * D * 4, KB = T * D * 4, VB = D * T * 4, PB = 128 * 32 * 4;
  static constexpr int PHASE1 = 2 * QB + 2 * KB, PHASE2 = 2 * VB + 4 * PB;
  static constexpr int REGION = PHASE1 > PHASE2 ? PHASE1 : PHASE2;
  static constexpr int SMEM = 1024 + REGION + 128;
  static constexpr uint32_t TCOLS = T + D <= 256 ? 256 : 512;
};

// Waits for `phase` of `bar`, bounded; every thread of the CTA calls it, and the outcome is
// made uniform across the CTA (a barrier, then the shared abort flag), so that the threads
// leave their loops together.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t phase, volatile int* abort, int* err, int code) {
  mbar_wait(bar, phase, abort, err, code);
  __syncthreads();
  return *abort == 0;
}

// Forward, one CTA per (batch entry, 128 query rows).
template <int T, int D>
__global__ void __launch_bounds__(TC_THREADS, 1) k_attn_fwd_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                             const float* __restrict__ v, const float* __restrict__ mask, float c, float fill,
                                                             int* err) {
  using L = FwdLayout<T, D>;
  constexpr int NQB = T / 128, NCH = T / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Qh = sm, *Ql = Qh + L::QB, *Kh = Ql + L::QB, *Kl = Kh + L::KB;  // phase 1
  uint8_t *Vh = sm, *Vl = Vh + L::VB, *P0 = Vl + L::VB;                     // phase 2: P buffers b: hi P0 + 2b PB, lo + PB
  uint64_t* bars = (uint64_t*)(sm + L::REGION);
  uint64_t *bar_s = bars, *bar_p = bars + 1, *bar_o = bars + 3, *bar_done = bars + 4;
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + tid;
  q += (z * T + r0) * D;
  k += z * T * D;
  v += z * T * D;

  if (tid == 0) {
    for (int b = 0; b < 5; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(L::TCOLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lanes = (uint32_t)(warp * 32) << 16;  // this warp's TMEM lane quarter
  const uint32_t S_t = tmem, O_t = tmem + T;

  // S = q k^T.
  stage(Qh, Ql, q, 128, D, D);
  stage(Kh, Kl, k, T, D, D);
  proxy_fence();
  __syncthreads();
  if (tid == 0) {
    fence_after();
    mma3(S_t, saddr(Qh), saddr(Ql), saddr(Kh), saddr(Kl), T, D, idesc_tf32(128, T), false);
    mma_commit(bar_s);
  }
  bool ok = cta_wait(bar_s, 0, abort, err, 21);
  fence_after();

  // Row statistics: the mask row as bits, the max, then the exp-sum in key order.
  uint32_t bits[NCH];
  float m = -INFINITY, sum = 0.0f;
  if (ok) {
    const float* mrow = mask + (long long)r * T;
#pragma unroll 1
    for (int ch = 0; ch < NCH; ++ch) {
      uint32_t x[32];
      tmem_ld32(S_t + lanes + ch * 32, x);
      uint32_t b = 0;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 mk = *(const float4*)(mrow + ch * 32 + j);
        b |= (mk.x != 0.0f ? 1u : 0u) << j | (mk.y != 0.0f ? 1u : 0u) << (j + 1) | (mk.z != 0.0f ? 1u : 0u) << (j + 2) |
             (mk.w != 0.0f ? 1u : 0u) << (j + 3);
      }
      bits[ch] = b;
#pragma unroll
      for (int j = 0; j < 32; ++j) m = nan_max(m, ((b >> j) & 1u) ? __uint_as_float(x[j]) / c : fill);
    }
#pragma unroll 1
    for (int ch = 0; ch < NCH; ++ch) {
      uint32_t x[32];
      tmem_ld32(S_t + lanes + ch * 32, x);
#pragma unroll
      for (int j = 0; j < 32; ++j) sum = sum + expf((((bits[ch] >> j) & 1u) ? __uint_as_float(x[j]) / c : fill) - m);
    }
  }
  fence_before();
  __syncthreads();

  // v^T into the freed operand space (the S products are complete).
  if (ok) {
    stage_t(Vh, Vl, v, T, D, D);
    proxy_fence();
  }
  __syncthreads();

  // O = P v, 32 keys at a time; P double-buffered in shared memory.
#pragma unroll 1
  for (int ch = 0; ch < NCH && ok; ++ch) {
    const int b = ch & 1;
    if (ch >= 2 && !cta_wait(&bar_p[b], (uint32_t)(((ch >> 1) - 1) & 1), abort, err, 22)) {
      ok = false;
      break;
    }
    fence_after();
    uint8_t* ph = P0 + 2 * b * L::PB;
    uint8_t* pl = ph + L::PB;
    uint32_t x[32];
    tmem_ld32(S_t + lanes + ch * 32, x);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float p[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) p[u] = expf((((bits[ch] >> (j + u)) & 1u) ? __uint_as_float(x[j + u]) / c : fill) - m) / sum;
      const uint32_t off = kmaj(128, tid, j);
      *(float4*)(ph + off) = make_float4(p[0], p[1], p[2], p[3]);
      *(float4*)(pl + off) = make_float4(tf32_lo(p[0]), tf32_lo(p[1]), tf32_lo(p[2]), tf32_lo(p[3]));
    }
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      const uint32_t vo = (uint32_t)(ch * D * 128);
      mma3(O_t, saddr(ph), saddr(pl), saddr(Vh) + vo, saddr(Vl) + vo, D, 32, idesc_tf32(128, D), ch > 0);
      mma_commit(&bar_p[b]);
    }
  }
  if (tid == 0) mma_commit(bar_o);
  if (ok) ok = cta_wait(bar_o, 0, abort, err, 23);
  fence_after();

  // O, m and s of row r.
  if (ok) {
    float* orow = out + ((z * T) + r) * (D + 2);
#pragma unroll 1
    for (int e0 = 0; e0 < D; e0 += 32) {
      uint32_t x[32];
      tmem_ld32(O_t + lanes + e0, x);
#pragma unroll
      for (int j = 0; j < 32; j += 2) *(float2*)(orow + e0 + j) = make_float2(__uint_as_float(x[j]), __uint_as_float(x[j + 1]));
    }
    *(float2*)(orow + D) = make_float2(m, sum);
  }

  // Teardown: every product issued has completed before the TMEM goes.
  fence_before();
  __syncthreads();
  if (tid == 0) {
    mma_commit(bar_done);
    unsigned long long t0 = now_ns();
    while (!mbar_try(bar_done, 0) && now_ns() - t0 < WAIT_LIMIT_NS) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TCOLS) : "memory");
  }
}

// Shared-memory plan of the backward kernels: phases a and b stage two 128-row operands each
// (hi and lo); phase c holds two transposed 128-column operands (dkdv) or one (dq) and the
// chunk tiles the epilogue writes (32 columns, hi and lo).
template <int D> struct BwdLayout {
  static constexpr int TB = 128 * D * 4;  // a 128 x D tile, or its transpose
  static constexpr int CB = 128 * 32 * 4; // a 128 x 32 chunk tile
  static constexpr int AB = 4 * TB;       // phases a, b
  static constexpr int DQ_C = 2 * TB + 4 * CB, KV_C = 4 * TB + 4 * CB;
  static constexpr int DQ_REGION = AB > DQ_C ? AB : DQ_C, KV_REGION = AB > KV_C ? AB : KV_C;
  static constexpr int DQ_SMEM = 1024 + DQ_REGION + 128, KV_SMEM = 1024 + KV_REGION + 3 * 128 * 4 + 128;
};

// Bounded wait on `bar` for its next phase; `count` tracks the phases already consumed.
__device__ __forceinline__ bool cta_next(uint64_t* bar, int& count, volatile int* abort, int* err, int code) {
  const bool ok = cta_wait(bar, (uint32_t)(count & 1), abort, err, code);
  ++count;
  return ok;
}

// dq, one CTA per (batch entry, 128 query rows), one thread per query row. Per half of the keys
// (128 keys): S = q k^T and dP = dO v^T into TMEM, then per 32-key chunk dS = P (dP - D) / c to
// shared memory and dq += dS k (k transposed, K-major over the keys).
template <int T, int D>
__global__ void __launch_bounds__(TC_THREADS, 1) k_attn_dq_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                            const float* __restrict__ v, const float* __restrict__ mask, const float* __restrict__ fwd,
                                                            const float* __restrict__ dout, float c, float fill, int* err) {
  using L = BwdLayout<D>;
  constexpr int NQB = T / 128, NH = T / 128, W = 3 * D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // phases a, b
  uint8_t *Kth = sm, *Ktl = Kth + L::TB, *C0 = Ktl + L::TB;              // phase c: k^T, dS chunks (buffer b: hi C0 + 2b CB)
  uint64_t* bars = (uint64_t*)(sm + L::DQ_REGION);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_done = bars + 4;  // bar_c: two buffers
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + tid;
  const float* qb = q + (z * T + r0) * D;
  const float* db = dout + (z * T + r0) * D;
  k += z * T * D;
  v += z * T * D;

  if (tid == 0) {
    for (int b = 0; b < 5; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(512u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot, lanes = (uint32_t)(warp * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, Q_t = tmem + 256;

  // Row r's statistics and D = dO . O.
  const float* fr = fwd + (z * T + r) * (D + 2);
  const float m = fr[D], sum = fr[D + 1];
  float Dr = 0.0f;
  {
    const float* dr = db + (long long)tid * D;
    for (int e = 0; e < D; e += 4) {
      const float4 a = *(const float4*)(dr + e);
      const float2 o0 = *(const float2*)(fr + e), o1 = *(const float2*)(fr + e + 2);
      Dr = Dr + a.x * o0.x;
      Dr = Dr + a.y * o0.y;
      Dr = Dr + a.z * o1.x;
      Dr = Dr + a.w * o1.y;
    }
  }
  const float* mrow = mask + (long long)r * T;
  bool ok = true;
  int na = 0, nb = 0, nc[2] = {0, 0};
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    // a: S = q k_h^T.
    stage(Ah, Al, qb, 128, D, D);
    stage(Bh, Bl, k + (long long)h * 128 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3(S_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), 128, D, idesc_tf32(128, 128), false);
      mma_commit(bar_a);
    }
    if (!(ok = cta_next(bar_a, na, abort, err, 31))) break;
    // b: dP = dO v_h^T.
    stage(Ah, Al, db, 128, D, D);
    stage(Bh, Bl, v + (long long)h * 128 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3(P_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), 128, D, idesc_tf32(128, 128), false);
      mma_commit(bar_b);
    }
    if (!(ok = cta_next(bar_b, nb, abort, err, 32))) break;
    fence_after();
    // c: k_h^T over the freed space, then dS chunk by chunk into dq.
    stage_t(Kth, Ktl, k + (long long)h * 128 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      const int b = ch & 1;
      if (ch >= 2 && !(ok = cta_next(&bar_c[b], nc[b], abort, err, 33))) break;
      fence_after();
      uint8_t* dh = C0 + 2 * b * L::CB;
      uint8_t* dl = dh + L::CB;
      uint32_t xs[32], xp[32];
      tmem_ld32(S_t + lanes + ch * 32, xs);
      tmem_ld32(P_t + lanes + ch * 32, xp);
      const int j0 = h * 128 + ch * 32;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 mk = *(const float4*)(mrow + j0 + j);
        const float mv[4] = {mk.x, mk.y, mk.z, mk.w};
        float ds[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool on = mv[u] != 0.0f;
          const float p = expf((on ? __uint_as_float(xs[j + u]) / c : fill) - m) / sum;
          ds[u] = on ? p * (__uint_as_float(xp[j + u]) - Dr) / c : 0.0f;
        }
        const uint32_t off = kmaj(128, tid, j);
        *(float4*)(dh + off) = make_float4(ds[0], ds[1], ds[2], ds[3]);
        *(float4*)(dl + off) = make_float4(tf32_lo(ds[0]), tf32_lo(ds[1]), tf32_lo(ds[2]), tf32_lo(ds[3]));
      }
      proxy_fence();
      fence_before();
      __syncthreads();
      if (tid == 0) {
        fence_after();
        const uint32_t ko = (uint32_t)(ch * D * 128);
        mma3(Q_t, saddr(dh), saddr(dl), saddr(Kth) + ko, saddr(Ktl) + ko, D, 32, idesc_tf32(128, D), h > 0 || ch > 0);
        mma_commit(&bar_c[b]);
      }
    }
    // The chunk products read k^T and dS from shared memory: they finish before the next half
    // stages over them (and before the next S overwrites the TMEM columns read above).
    for (int b = 0; b < 2 && ok; ++b)
      if (!(ok = cta_next(&bar_c[b], nc[b], abort, err, 34))) break;
    fence_after();
  }
  fence_after();
  if (ok) {
    float* g = out + (z * T + r) * W;
#pragma unroll 1
    for (int e0 = 0; e0 < D; e0 += 32) {
      uint32_t x[32];
      tmem_ld32(Q_t + lanes + e0, x);
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *(float4*)(g + e0 + j) = make_float4(__uint_as_float(x[j]), __uint_as_float(x[j + 1]), __uint_as_float(x[j + 2]), __uint_as_float(x[j + 3]));
    }
  }
  fence_before();
  __syncthreads();
  if (tid == 0) {
    mma_commit(bar_done);
    unsigned long long t0 = now_ns();
    while (!mbar_try(bar_done, 0) && now_ns() - t0 < WAIT_LIMIT_NS) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

// dk and dv, one CTA per (batch entry, 128 keys), one thread per key row. Per half of the
// queries (128 queries): S^T = k q^T and dP^T = v dO^T into TMEM, then per 32-query chunk P^T and
// dS^T to shared memory, dv += P^T dO and dk += dS^T q (dO and q transposed, K-major over the
// queries). The queries' statistics (max, exp-sum, D = dO . O) sit in shared memory.
template <int T, int D>
__global__ void __launch_bounds__(TC_THREADS, 1) k_attn_dkdv_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                              const float* __restrict__ v, const float* __restrict__ mask,
                                                              const float* __restrict__ fwd, const float* __restrict__ dout, float c, float fill,
                                                              int* err) {
  using L = BwdLayout<D>;
  constexpr int NKB = T / 128, NH = T / 128, W = 3 * D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // phases a, b
  uint8_t *Qth = sm, *Qtl = Qth + L::TB, *Oth = Qtl + L::TB, *Otl = Oth + L::TB;  // phase c: q^T, dO^T
  uint8_t *Ph = Otl + L::TB, *Pl = Ph + L::CB, *Dh = Pl + L::CB, *Dl = Dh + L::CB;  // P^T and dS^T chunks
  float* stats = (float*)(sm + L::KV_REGION);  // [3][128]: max, exp-sum, D of the half's queries
  uint64_t* bars = (uint64_t*)(stats + 3 * 128);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_done = bars + 3;
  uint32_t* tslot = (uint32_t*)(bars + 4);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const long long z = blockIdx.x / NKB;
  const int j0 = (int)(blockIdx.x - z * NKB) * 128, j = j0 + tid;
  const float* kb = k + (z * T + j0) * D;
  const float* vb = v + (z * T + j0) * D;
  q += z * T * D;
  dout += z * T * D;
  fwd += z * T * (D + 2);

  if (tid == 0) {
    for (int b = 0; b < 4; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(512u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot, lanes = (uint32_t)(warp * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, V_t = tmem + 256, K_t = tmem + 256 + D;

  bool ok = true;
  int na = 0, nb = 0, nc = 0;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    const int q0 = h * 128;
    // The half's query statistics: thread i takes query q0 + i.
    {
      const float* fr = fwd + (long long)(q0 + tid) * (D + 2);
      const float* dr = dout + (long long)(q0 + tid) * D;
      float Dq = 0.0f;
      for (int e = 0; e < D; e += 4) {
        const float4 a = *(const float4*)(dr + e);
        const float2 o0 = *(const float2*)(fr + e), o1 = *(const float2*)(fr + e + 2);
        Dq = Dq + a.x * o0.x;
        Dq = Dq + a.y * o0.y;
        Dq = Dq + a.z * o1.x;
        Dq = Dq + a.w * o1.y;
      }
      stats[tid] = fr[D];
      stats[128 + tid] = fr[D + 1];
      stats[256 + tid] = Dq;
    }
    // a: S^T = k q_h^T.
    stage(Ah, Al, kb, 128, D, D);
    stage(Bh, Bl, q + (long long)q0 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3(S_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), 128, D, idesc_tf32(128, 128), false);
      mma_commit(bar_a);
    }
    if (!(ok = cta_next(bar_a, na, abort, err, 41))) break;
    // b: dP^T = v dO_h^T.
    stage(Ah, Al, vb, 128, D, D);
    stage(Bh, Bl, dout + (long long)q0 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3(P_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), 128, D, idesc_tf32(128, 128), false);
      mma_commit(bar_b);
    }
    if (!(ok = cta_next(bar_b, nb, abort, err, 42))) break;
    fence_after();
    // c: q_h^T and dO_h^T over the freed space, then P^T and dS^T chunk by chunk.
    stage_t(Qth, Qtl, q + (long long)q0 * D, 128, D, D);
    stage_t(Oth, Otl, dout + (long long)q0 * D, 128, D, D);
    proxy_fence();
    __syncthreads();
#pragma unroll 1
    for (int ch = 0; ch < 4; ++ch) {
      if (ch > 0 && !(ok = cta_next(bar_c, nc, abort, err, 43))) break;
      fence_after();
      uint32_t xs[32], xp[32];
      tmem_ld32(S_t + lanes + ch * 32, xs);
      tmem_ld32(P_t + lanes + ch * 32, xp);
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float pv[4], dv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int rl = ch * 32 + i + u, rq = q0 + rl;
          const bool on = mask[(long long)rq * T + j] != 0.0f;
          const float p = expf((on ? __uint_as_float(xs[i + u]) / c : fill) - stats[rl]) / stats[128 + rl];
          pv[u] = p;
          dv[u] = on ? p * (__uint_as_float(xp[i + u]) - stats[256 + rl]) / c : 0.0f;
        }
        const uint32_t off = kmaj(128, tid, i);
        *(float4*)(Ph + off) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        *(float4*)(Pl + off) = make_float4(tf32_lo(pv[0]), tf32_lo(pv[1]), tf32_lo(pv[2]), tf32_lo(pv[3]));
        *(float4*)(Dh + off) = make_float4(dv[0], dv[1], dv[2], dv[3]);
        *(float4*)(Dl + off) = make_float4(tf32_lo(dv[0]), tf32_lo(dv[1]), tf32_lo(dv[2]), tf32_lo(dv[3]));
      }
      proxy_fence();
      fence_before();
      __syncthreads();
      if (tid == 0) {
        fence_after();
        const uint32_t qo = (uint32_t)(ch * D * 128);
        const bool acc = h > 0 || ch > 0;
        mma3(V_t, saddr(Ph), saddr(Pl), saddr(Oth) + qo, saddr(Otl) + qo, D, 32, idesc_tf32(128, D), acc);
        mma3(K_t, saddr(Dh), saddr(Dl), saddr(Qth) + qo, saddr(Qtl) + qo, D, 32, idesc_tf32(128, D), acc);
        mma_commit(bar_c);
      }
    }
    // The last chunk's products finish before the stats, tiles and TMEM columns are reused.
    if (ok) ok = cta_next(bar_c, nc, abort, err, 44);
    fence_after();
  }
  fence_after();
  if (ok) {
    float* g = out + (z * T + j) * W;
#pragma unroll 1
    for (int e0 = 0; e0 < D; e0 += 32) {
      uint32_t x[32], y[32];
      tmem_ld32(K_t + lanes + e0, x);
      tmem_ld32(V_t + lanes + e0, y);
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        *(float4*)(g + D + e0 + u) = make_float4(__uint_as_float(x[u]), __uint_as_float(x[u + 1]), __uint_as_float(x[u + 2]), __uint_as_float(x[u + 3]));
        *(float4*)(g + 2 * D + e0 + u) =
            make_float4(__uint_as_float(y[u]), __uint_as_float(y[u + 1]), __uint_as_float(y[u + 2]), __uint_as_float(y[u + 3]));
      }
    }
  }
  fence_before();
  __syncthreads();
  if (tid == 0) {
    mma_commit(bar_done);
    unsigned long long t0 = now_ns();
    while (!mbar_try(bar_done, 0) && now_ns() - t0 < WAIT_LIMIT_NS) {
    }
  }
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

template <int T, int D> void set_smem(void (*kern)(float*, const float*, const float*, const float*, const float*, float, float, int*)) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<T, D>::SMEM);
}

template <int T, int D> void launch_fwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const AttnShape& a, int* err,
                                           cudaStream_t s) {
  const long long blocks = a.batch * (T / 128);
  k_attn_fwd_tc<T, D><<<(unsigned)blocks, TC_THREADS, FwdLayout<T, D>::SMEM, s>>>(out, q, k, v, mask, a.c, a.fill, err);
}

template <int T, int D> void set_smem_bwd() {
  cudaFuncSetAttribute(k_attn_dq_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<D>::DQ_SMEM);
  cudaFuncSetAttribute(k_attn_dkdv_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<D>::KV_SMEM);
}

template <int T, int D> void launch_bwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd,
                                           const float* dout, const AttnShape& a, int* err, cudaStream_t s) {
  const unsigned blocks = (unsigned)(a.batch * (T / 128));
  k_attn_dq_tc<T, D><<<blocks, TC_THREADS, BwdLayout<D>::DQ_SMEM, s>>>(out, q, k, v, mask, fwd, dout, a.c, a.fill, err);
  k_attn_dkdv_tc<T, D><<<blocks, TC_THREADS, BwdLayout<D>::KV_SMEM, s>>>(out, q, k, v, mask, fwd, dout, a.c, a.fill, err);
}

}  // namespace

void attention_init() {
  static std::once_flag once;
  std::call_once(once, [] {
    set_smem<128, 32>(k_attn_fwd_tc<128, 32>);
    set_smem<128, 64>(k_attn_fwd_tc<128, 64>);
    set_smem<256, 32>(k_attn_fwd_tc<256, 32>);
    set_smem<256, 64>(k_attn_fwd_tc<256, 64>);
    set_smem_bwd<128, 32>();
    set_smem_bwd<128, 64>();
    set_smem_bwd<256, 32>();
    set_smem_bwd<256, 64>();
  });
}

bool attention_tc_supported(const AttnShape& a) {
  return (a.t == 128 || a.t == 256) && (a.d == 32 || a.d == 64) && a.dv == a.d && a.batch > 0 && a.batch * (a.t / 128) < (1LL << 31);
}

void attention_fwd(float* out, const float* q, const float* k, const float* v, const float* mask, const AttnShape& a, int* error, cudaStream_t s) {
  if (a.batch == 0) return;
  if (attention_tc_supported(a)) {
    if (a.t == 128 && a.d == 32) return launch_fwd_tc<128, 32>(out, q, k, v, mask, a, error, s);
    if (a.t == 128) return launch_fwd_tc<128, 64>(out, q, k, v, mask, a, error, s);
    if (a.d == 32) return launch_fwd_tc<256, 32>(out, q, k, v, mask, a, error, s);
    return launch_fwd_tc<256, 64>(out, q, k, v, mask, a, error, s);
  }
  const long long rows = a.batch * a.t;
  k_attn_fwd_simt<<<(unsigned)((rows + 3) / 4), 128, 4 * a.t * sizeof(float), s>>>(out, q, k, v, mask, rows, a.t, a.d, a.dv, a.c, a.fill);
}

void attention_bwd(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd, const float* dout,
                   const AttnShape& a, int* error, cudaStream_t s) {
  if (a.batch == 0) return;
  if (attention_tc_supported(a)) {
    if (a.t == 128 && a.d == 32) return launch_bwd_tc<128, 32>(out, q, k, v, mask, fwd, dout, a, error, s);
    if (a.t == 128) return launch_bwd_tc<128, 64>(out, q, k, v, mask, fwd, dout, a, error, s);
    if (a.d == 32) return launch_bwd_tc<256, 32>(out, q, k, v, mask, fwd, dout, a, error, s);
    return launch_bwd_tc<256, 64>(out, q, k, v, mask, fwd, dout, a, error, s);
  }
  const long long rows = a.batch * a.t;
  const unsigned blocks = (unsigned)((rows + 3) / 4);
  k_attn_dq_simt<<<blocks, 128, 4 * a.t * sizeof(float), s>>>(out, q, k, v, mask, fwd, dout, rows, a.t, a.d, a.dv, a.c, a.fill);
  k_attn_dkdv_simt<<<blocks, 128, 8 * a.t * sizeof(float), s>>>(out, q, k, v, mask, fwd, dout, rows, a.t, a.d, a.dv, a.c, a.fill);
}

}  // namespace rgc
