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

// Byte offset of element (row, k) in a K-major tile of R rows whose K extent is cut into 32-wide
// blocks (R x 128 bytes each): 8-row groups of 1024 bytes, 128 bytes per row, and the row's
// 16-byte chunk (k % 32) / 4 stored at chunk position ((k % 32) / 4) ^ (row % 8) — the 128-byte
// swizzle that desc_k describes (the layout TMA's SWIZZLE_128B writes for gemm_tc.cu).
__device__ __forceinline__ uint32_t kmaj(int R, int row, int k) {
  return (uint32_t)((k >> 5) * R * 128 + (row >> 3) * 1024 + (row & 7) * 128 + ((((k & 31) >> 2) ^ (row & 7)) << 4) + ((k & 3) << 2));
}

__device__ __forceinline__ float tf32_lo(float x) { return x - tf32_trunc(x); }

// Rows [0, R) x columns [0, K) of a row-major global block (row stride `ld` floats, 16-byte
// aligned rows) into K-major hi / lo tiles. Each thread moves four 16-byte vectors at a time,
// all four loads issued before the first store.
__device__ __forceinline__ void stage(uint8_t* hi, uint8_t* lo, const float* __restrict__ src, int R, int K, long long ld) {
  const int k4 = K >> 2, n = R * k4, step = blockDim.x;
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * step) {
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * step;
      if (i < n) {
        const int row = i / k4, col = (i - row * k4) << 2;
        x[u] = *(const float4*)(src + row * ld + col);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * step;
      if (i < n) {
        const int row = i / k4, col = (i - row * k4) << 2;
        const uint32_t off = kmaj(R, row, col);
        *(float4*)(hi + off) = x[u];
        *(float4*)(lo + off) = make_float4(tf32_lo(x[u].x), tf32_lo(x[u].y), tf32_lo(x[u].z), tf32_lo(x[u].w));
      }
    }
  }
}

// The transpose of a row-major global block: source rows [0, Rs) become the tile's K index and
// source columns [0, Cs) its rows (a K-major tile of Cs rows over K = Rs). Each thread takes a
// 4 x 4 block (source rows j..j+3, columns e..e+3), transposes it in registers and writes four
// 16-byte vectors (tile rows e..e+3, K = j..j+3). Rs and Cs are multiples of 4.
__device__ __forceinline__ void stage_t(uint8_t* hi, uint8_t* lo, const float* __restrict__ src, int Rs, int Cs, long long ld) {
  const int c4 = Cs >> 2, n = (Rs >> 2) * c4;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int jb = i / c4, e = (i - jb * c4) << 2, j = jb << 2;
    float4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = *(const float4*)(src + (long long)(j + u) * ld + e);
    const float4 t[4] = {make_float4(x[0].x, x[1].x, x[2].x, x[3].x), make_float4(x[0].y, x[1].y, x[2].y, x[3].y),
                         make_float4(x[0].z, x[1].z, x[2].z, x[3].z), make_float4(x[0].w, x[1].w, x[2].w, x[3].w)};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t off = kmaj(Cs, e + u, j);
      *(float4*)(hi + off) = t[u];
      *(float4*)(lo + off) = make_float4(tf32_lo(t[u].x), tf32_lo(t[u].y), tf32_lo(t[u].z), tf32_lo(t[u].w));
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

// Waits for `phase` of `bar`, bounded; every thread of the CTA calls it, and the outcome is
// made uniform across the CTA (a barrier, then the shared abort flag), so that the threads
// leave their loops together.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t phase, volatile int* abort, int* err, int code) {
  mbar_wait(bar, phase, abort, err, code);
  __syncthreads();
  return *abort == 0;
}

constexpr int FWD_THREADS = 512;

template <int T, int D> struct FwdLayout {
  static constexpr int QB = 128 * D * 4, KB = T * D * 4;
  static constexpr int VB = D * 128 * 4;   // v^T of one half of the keys: D rows over 128 keys
  static constexpr int EB = 128 * 32 * 4;  // one 32-key chunk of E
  static constexpr int PHASE1 = 2 * QB + 2 * KB, PHASE2 = 2 * VB + 8 * EB;
  static constexpr int REGION = PHASE1 > PHASE2 ? PHASE1 : PHASE2;
  static constexpr int SMEM = 1024 + REGION + 2 * 4 * 128 * 4 + 128;
  static constexpr uint32_t TCOLS = T + D <= 256 ? 256 : 512;
};

// Forward, one CTA of 16 warps per (batch entry, 128 query rows). Warp w reads TMEM lanes
// 32 (w % 4) .. +31 (query rows) and, as group g = w / 4, the key chunk g of every half of
// 128 keys, so the four warps of a row share its 32-column chunks. Pass 1 gives each row's
// maximum (partial maxima combined through shared memory); then per half of the keys
// E = exp(Z - m) goes to shared memory as four 32-key chunks (hi and lo) beside v^T of the
// half, and O += E v accumulates in TMEM. O is divided by the row's exp-sum at the end.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_fwd_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                              const float* __restrict__ v, const float* __restrict__ mask, float inv_c, float fill,
                                                              int* err) {
  using L = FwdLayout<T, D>;
  constexpr int NQB = T / 128, NH = T / 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Qh = sm, *Ql = Qh + L::QB, *Kh = Ql + L::QB, *Kl = Kh + L::KB;  // phase 1
  uint8_t *Vh = sm, *Vl = Vh + L::VB, *E0 = Vl + L::VB;                     // phase 2: chunk g at E0 + 2 g EB (hi), + EB (lo)
  float* part = (float*)(sm + L::REGION);                                   // [2][4][128]: partial max, partial sum
  uint64_t* bars = (uint64_t*)(part + 2 * 4 * 128);
  uint64_t *bar_s = bars, *bar_o = bars + 1, *bar_done = bars + 2;
  uint32_t* tslot = (uint32_t*)(bars + 3);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;  // this thread's query row within the block
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + row;
  q += (z * T + r0) * D;
  k += z * T * D;
  v += z * T * D;

  if (tid == 0) {
    for (int b = 0; b < 3; ++b) mbar_init(&bars[b], 1);
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
  const uint32_t lanes = (uint32_t)(lq * 32) << 16;
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

  // Pass 1: the mask bits of this thread's chunks and the row maximum.
  const float* mrow = mask + (long long)r * T;
  uint32_t bits[NH];
  float m = -INFINITY;
  if (ok) {
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const int c0 = h * 128 + g * 32;
      uint32_t x[32];
      tmem_ld32(S_t + lanes + c0, x);
      uint32_t b = 0;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 mk = *(const float4*)(mrow + c0 + j);
        b |= (mk.x != 0.0f ? 1u : 0u) << j | (mk.y != 0.0f ? 1u : 0u) << (j + 1) | (mk.z != 0.0f ? 1u : 0u) << (j + 2) |
             (mk.w != 0.0f ? 1u : 0u) << (j + 3);
      }
      bits[h] = b;
#pragma unroll
      for (int j = 0; j < 32; ++j) m = nan_max(m, ((b >> j) & 1u) ? __uint_as_float(x[j]) * inv_c : fill);
    }
    part[g * 128 + row] = m;
  }
  __syncthreads();
  if (ok) m = nan_max(nan_max(part[row], part[128 + row]), nan_max(part[256 + row], part[384 + row]));

  // Per half of the keys: v^T of the half and the half's E chunks in shared memory, then
  // O += E v (the S products are complete, so their operand space is free).
  float sum = 0.0f;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    if (h > 0 && !(ok = cta_wait(bar_o, (uint32_t)((h - 1) & 1), abort, err, 22))) break;
    stage_t(Vh, Vl, v + (long long)h * 128 * D, 128, D, D);
    const int c0 = h * 128 + g * 32;
    uint32_t x[32];
    tmem_ld32(S_t + lanes + c0, x);
    uint8_t* eh = E0 + 2 * g * L::EB;
    uint8_t* el = eh + L::EB;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float e[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        e[u] = __expf((((bits[h] >> (j + u)) & 1u) ? __uint_as_float(x[j + u]) * inv_c : fill) - m);
        sum = sum + e[u];
      }
      const uint32_t off = kmaj(128, row, j);
      *(float4*)(eh + off) = make_float4(e[0], e[1], e[2], e[3]);
      *(float4*)(el + off) = make_float4(tf32_lo(e[0]), tf32_lo(e[1]), tf32_lo(e[2]), tf32_lo(e[3]));
    }
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint8_t* ch = E0 + 2 * cc * L::EB;
        const uint32_t vo = (uint32_t)(cc * D * 128);
        mma3(O_t, saddr(ch), saddr(ch + L::EB), saddr(Vh) + vo, saddr(Vl) + vo, D, 32, idesc_tf32(128, D), h > 0 || cc > 0);
      }
      mma_commit(bar_o);
    }
  }
  if (ok) ok = cta_wait(bar_o, (uint32_t)((NH - 1) & 1), abort, err, 23);
  fence_after();
  if (ok) part[512 + g * 128 + row] = sum;
  __syncthreads();

  // O / s, m and s of row r: group g writes O columns [32 g, 32 g + 32).
  if (ok) {
    const float s4 = (part[512 + row] + part[640 + row]) + (part[768 + row] + part[896 + row]);
    float* orow = out + ((z * T) + r) * (D + 2);
    if (g * 32 < D) {
      uint32_t x[32];
      tmem_ld32(O_t + lanes + g * 32, x);
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *(float2*)(orow + g * 32 + j) = make_float2(__uint_as_float(x[j]) / s4, __uint_as_float(x[j + 1]) / s4);
    }
    if (g == 0) *(float2*)(orow + D) = make_float2(m, s4);
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

// Shared-memory plan of the backward kernels: phases a and b stage two 128-row operands (hi and
// lo); phase c holds one transposed operand (128 columns) and the four 32-column chunk tiles
// the four warp groups write.
template <int D> struct BwdLayout {
  static constexpr int TB = 128 * D * 4;  // a 128 x D tile, or its transpose
  static constexpr int CB = 128 * 32 * 4; // a 128 x 32 chunk tile
  static constexpr int AB = 4 * TB, CPH = 2 * TB + 8 * CB;
  static constexpr int REGION = AB > CPH ? AB : CPH;
  static constexpr int SMEM = 1024 + REGION + 3 * 128 * 4 + 128;
};

// Bounded wait on `bar` for its next phase; `count` tracks the phases already consumed.
__device__ __forceinline__ bool cta_next(uint64_t* bar, int& count, volatile int* abort, int* err, int code) {
  const bool ok = cta_wait(bar, (uint32_t)(count & 1), abort, err, code);
  ++count;
  return ok;
}

// The mask bits of 32 consecutive elements of a row.
__device__ __forceinline__ uint32_t mask_bits(const float* m) {
  uint32_t b = 0;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 mk = *(const float4*)(m + j);
    b |= (mk.x != 0.0f ? 1u : 0u) << j | (mk.y != 0.0f ? 1u : 0u) << (j + 1) | (mk.z != 0.0f ? 1u : 0u) << (j + 2) | (mk.w != 0.0f ? 1u : 0u) << (j + 3);
  }
  return b;
}

__device__ __forceinline__ void put_chunk(uint8_t* hi, uint8_t* lo, int row, const float (&x)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const uint32_t off = kmaj(128, row, j);
    *(float4*)(hi + off) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
    *(float4*)(lo + off) = make_float4(tf32_lo(x[j]), tf32_lo(x[j + 1]), tf32_lo(x[j + 2]), tf32_lo(x[j + 3]));
  }
}

__device__ __forceinline__ void tc_teardown(uint64_t* bar_done, uint32_t tmem, uint32_t cols) {
  fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mma_commit(bar_done);
    unsigned long long t0 = now_ns();
    while (!mbar_try(bar_done, 0) && now_ns() - t0 < WAIT_LIMIT_NS) {
    }
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
  }
}

// dq, one CTA of 16 warps per (batch entry, 128 query rows); warp w reads TMEM lanes 32 (w % 4)
// (query rows) and, as group g = w / 4, key chunk g of each half. Per half of the keys (128):
// S = q k^T and dP = dO v^T into TMEM, then k^T of the half and the four dS chunks in shared
// memory, and dq += dS k.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_dq_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                             const float* __restrict__ v, const float* __restrict__ mask, const float* __restrict__ fwd,
                                                             const float* __restrict__ dout, float inv_c, float fill, int* err) {
  using L = BwdLayout<D>;
  constexpr int NQB = T / 128, NH = T / 128, W = 3 * D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // phases a, b
  uint8_t *Th = sm, *Tl = Th + L::TB, *C0 = Tl + L::TB;                  // phase c: k^T, chunk g at C0 + 2 g CB
  uint64_t* bars = (uint64_t*)(sm + L::REGION + 3 * 128 * 4);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_done = bars + 3;
  uint32_t* tslot = (uint32_t*)(bars + 4);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + row;
  const float* qb = q + (z * T + r0) * D;
  const float* db = dout + (z * T + r0) * D;
  k += z * T * D;
  v += z * T * D;

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
  const uint32_t tmem = *tslot, lanes = (uint32_t)(lq * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, Q_t = tmem + 256;

  // Row r's statistics and D = dO . O.
  const float* fr = fwd + (z * T + r) * (D + 2);
  const float m = fr[D], inv_sum = 1.0f / fr[D + 1];
  float Dr = 0.0f;
  {
    const float* dr = db + (long long)row * D;
    for (int e = 0; e < D; e += 4) {
      const float4 a4 = *(const float4*)(dr + e);
      const float2 o0 = *(const float2*)(fr + e), o1 = *(const float2*)(fr + e + 2);
      Dr = Dr + a4.x * o0.x;
      Dr = Dr + a4.y * o0.y;
      Dr = Dr + a4.z * o1.x;
      Dr = Dr + a4.w * o1.y;
    }
  }
  const float* mrow = mask + (long long)r * T;
  bool ok = true;
  int na = 0, nb = 0, nc = 0;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    // a: S = q k_h^T (the previous half's products are complete).
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
    // c: k_h^T, and this group's dS chunk.
    stage_t(Th, Tl, k + (long long)h * 128 * D, 128, D, D);
    {
      uint32_t xs[32], xp[32];
      tmem_ld32(S_t + lanes + g * 32, xs);
      tmem_ld32(P_t + lanes + g * 32, xp);
      const uint32_t bits = mask_bits(mrow + h * 128 + g * 32);
      float ds[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const bool on = (bits >> j) & 1u;
        const float p = __expf((on ? __uint_as_float(xs[j]) * inv_c : fill) - m) * inv_sum;
        ds[j] = on ? p * (__uint_as_float(xp[j]) - Dr) * inv_c : 0.0f;
      }
      put_chunk(C0 + 2 * g * L::CB, C0 + (2 * g + 1) * L::CB, row, ds);
    }
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const uint32_t ko = (uint32_t)(cc * D * 128);
        uint8_t* ch = C0 + 2 * cc * L::CB;
        mma3(Q_t, saddr(ch), saddr(ch + L::CB), saddr(Th) + ko, saddr(Tl) + ko, D, 32, idesc_tf32(128, D), h > 0 || cc > 0);
      }
      mma_commit(bar_c);
    }
    if (!(ok = cta_next(bar_c, nc, abort, err, 33))) break;
    fence_after();
  }
  if (ok && g * 32 < D) {
    float* gq = out + (z * T + r) * W + g * 32;
    uint32_t x[32];
    tmem_ld32(Q_t + lanes + g * 32, x);
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *(float4*)(gq + j) = make_float4(__uint_as_float(x[j]), __uint_as_float(x[j + 1]), __uint_as_float(x[j + 2]), __uint_as_float(x[j + 3]));
  }
  tc_teardown(bar_done, tmem, 512u);
}

// dk and dv, one CTA of 16 warps per (batch entry, 128 keys); warp w reads TMEM lanes 32 (w % 4)
// (key rows) and, as group g = w / 4, query chunk g of each half. Per half of the queries
// (128): S^T = k q^T and dP^T = v dO^T into TMEM; then dO^T of the half and the four P^T chunks
// in shared memory, dv += P^T dO; then q^T and the four dS^T chunks (kept in registers
// meanwhile), dk += dS^T q. The half's query statistics (max, 1 / exp-sum, D) sit in shared memory.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_dkdv_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, const float* __restrict__ mask,
                                                               const float* __restrict__ fwd, const float* __restrict__ dout, float inv_c, float fill,
                                                               int* err) {
  using L = BwdLayout<D>;
  constexpr int NKB = T / 128, NH = T / 128, W = 3 * D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // phases a, b
  uint8_t *Th = sm, *Tl = Th + L::TB, *C0 = Tl + L::TB;                  // phase c
  float* stats = (float*)(sm + L::REGION);  // [3][128]
  uint64_t* bars = (uint64_t*)(stats + 3 * 128);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_done = bars + 3;
  uint32_t* tslot = (uint32_t*)(bars + 4);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;  // key row within the block
  const long long z = blockIdx.x / NKB;
  const int j0 = (int)(blockIdx.x - z * NKB) * 128, j = j0 + row;
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
  const uint32_t tmem = *tslot, lanes = (uint32_t)(lq * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, V_t = tmem + 256, K_t = tmem + 256 + D;

  bool ok = true;
  int na = 0, nb = 0, nc = 0;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    const int q0 = h * 128;
    // The half's query statistics (the previous half's readers finished at its last wait).
    if (tid < 128) {
      const float* fr = fwd + (long long)(q0 + tid) * (D + 2);
      const float* dr = dout + (long long)(q0 + tid) * D;
      float Dq = 0.0f;
      for (int e = 0; e < D; e += 4) {
        const float4 a4 = *(const float4*)(dr + e);
        const float2 o0 = *(const float2*)(fr + e), o1 = *(const float2*)(fr + e + 2);
        Dq = Dq + a4.x * o0.x;
        Dq = Dq + a4.y * o0.y;
        Dq = Dq + a4.z * o1.x;
        Dq = Dq + a4.w * o1.y;
      }
      stats[tid] = fr[D];
      stats[128 + tid] = 1.0f / fr[D + 1];
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
    // c1: dO_h^T and this group's P^T chunk (query columns q0 + 32 g ..).
    stage_t(Th, Tl, dout + (long long)q0 * D, 128, D, D);
    uint32_t qbits = 0;  // the mask bits of this key column over the chunk's queries
#pragma unroll 8
    for (int i = 0; i < 32; ++i) qbits |= (mask[(long long)(q0 + g * 32 + i) * T + j] != 0.0f ? 1u : 0u) << i;
    {
      uint32_t xs[32];
      tmem_ld32(S_t + lanes + g * 32, xs);
      float pv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int rl = g * 32 + i;
        pv[i] = __expf((((qbits >> i) & 1u) ? __uint_as_float(xs[i]) * inv_c : fill) - stats[rl]) * stats[128 + rl];
      }
      put_chunk(C0 + 2 * g * L::CB, C0 + (2 * g + 1) * L::CB, row, pv);
    }
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const uint32_t qo = (uint32_t)(cc * D * 128);
        uint8_t* ch = C0 + 2 * cc * L::CB;
        mma3(V_t, saddr(ch), saddr(ch + L::CB), saddr(Th) + qo, saddr(Tl) + qo, D, 32, idesc_tf32(128, D), h > 0 || cc > 0);
      }
      mma_commit(bar_c);
    }
    if (!(ok = cta_next(bar_c, nc, abort, err, 43))) break;
    // c2: q_h^T and the dS^T chunks (P^T recomputed from the scores still in TMEM).
    stage_t(Th, Tl, q + (long long)q0 * D, 128, D, D);
    {
      uint32_t xs[32], xp[32];
      tmem_ld32(S_t + lanes + g * 32, xs);
      tmem_ld32(P_t + lanes + g * 32, xp);
      float dsv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int rl = g * 32 + i;
        const bool on = (qbits >> i) & 1u;
        const float p = __expf((on ? __uint_as_float(xs[i]) * inv_c : fill) - stats[rl]) * stats[128 + rl];
        dsv[i] = on ? p * (__uint_as_float(xp[i]) - stats[256 + rl]) * inv_c : 0.0f;
      }
      put_chunk(C0 + 2 * g * L::CB, C0 + (2 * g + 1) * L::CB, row, dsv);
    }
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const uint32_t qo = (uint32_t)(cc * D * 128);
        uint8_t* ch = C0 + 2 * cc * L::CB;
        mma3(K_t, saddr(ch), saddr(ch + L::CB), saddr(Th) + qo, saddr(Tl) + qo, D, 32, idesc_tf32(128, D), h > 0 || cc > 0);
      }
      mma_commit(bar_c);
    }
    if (!(ok = cta_next(bar_c, nc, abort, err, 44))) break;
    fence_after();
  }
  if (ok && g * 32 < D) {
    float* gk = out + (z * T + j) * W;
    uint32_t x[32], y[32];
    tmem_ld32(K_t + lanes + g * 32, x);
    tmem_ld32(V_t + lanes + g * 32, y);
#pragma unroll
    for (int u = 0; u < 32; u += 4) {
      *(float4*)(gk + D + g * 32 + u) = make_float4(__uint_as_float(x[u]), __uint_as_float(x[u + 1]), __uint_as_float(x[u + 2]), __uint_as_float(x[u + 3]));
      *(float4*)(gk + 2 * D + g * 32 + u) = make_float4(__uint_as_float(y[u]), __uint_as_float(y[u + 1]), __uint_as_float(y[u + 2]), __uint_as_float(y[u + 3]));
    }
  }
  tc_teardown(bar_done, tmem, 512u);
}

template <int T, int D> void set_smem(void (*kern)(float*, const float*, const float*, const float*, const float*, float, float, int*)) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<T, D>::SMEM);
}

template <int T, int D> void launch_fwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const AttnShape& a, int* err,
                                           cudaStream_t s) {
  const long long blocks = a.batch * (T / 128);
  k_attn_fwd_tc<T, D><<<(unsigned)blocks, FWD_THREADS, FwdLayout<T, D>::SMEM, s>>>(out, q, k, v, mask, 1.0f / a.c, a.fill, err);
}

template <int T, int D> void set_smem_bwd() {
  cudaFuncSetAttribute(k_attn_dq_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<D>::SMEM);
  cudaFuncSetAttribute(k_attn_dkdv_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<D>::SMEM);
}

template <int T, int D> void launch_bwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd,
                                           const float* dout, const AttnShape& a, int* err, cudaStream_t s) {
  const unsigned blocks = (unsigned)(a.batch * (T / 128));
  k_attn_dq_tc<T, D><<<blocks, FWD_THREADS, BwdLayout<D>::SMEM, s>>>(out, q, k, v, mask, fwd, dout, 1.0f / a.c, a.fill, err);
  k_attn_dkdv_tc<T, D><<<blocks, FWD_THREADS, BwdLayout<D>::SMEM, s>>>(out, q, k, v, mask, fwd, dout, 1.0f / a.c, a.fill, err);
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
