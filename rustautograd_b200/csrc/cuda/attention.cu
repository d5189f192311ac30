// Fused attention (attention.cuh) on sm_100a.
//
// Tensor-core path (T = 128 or 256, d = dv = 32 or 64): 3xTF32 products on tcgen05 with fp32
// accumulators in TMEM, as in gemm_tc.cu (hi = the raw fp32 value, which the tensor core reads as
// TF32; lo = x - trunc_tf32(x); A B = A_hi B_hi + A_hi B_lo + A_lo B_hi). Operand tiles are staged
// in shared memory by the CTA's own threads, which write hi and lo in the K-major 128-byte-swizzle
// layout the MMA descriptors read (a transposed operand is written transposed, so every operand is
// K-major). One CTA of 16 warps takes 128 rows (queries, or keys for dk / dv) of one batch entry:
// warp w reads TMEM lanes 32 (w % 4) .. + 31 and, as group w / 4, one 32-column chunk of every
// 128 columns, so a row's four warps share its chunks.
//   forward   S = q k^T into TMEM (T columns); pass 1 gives each row's max; then per half of the
//             keys E = exp(Z - m) replaces S in TMEM (hi; lo in a TMEM buffer) and O += E v
//             takes E from TMEM as the product's A operand; O / s, m and s leave as the block's
//             contiguous packed rows.
//   backward  two kernels, each recomputing the scores: k_attn_dq_tc (query rows) forms dS per
//             half of the keys and accumulates dq = dS k; k_attn_dkdv_tc (key rows) works on the
//             transposes, forming P^T and dS^T and accumulating dv = P^T dO and dk = dS^T q.
//             dS, P^T and dS^T, like E, are A operands in TMEM. D = rowsum(dO * O) comes from
//             the forward's O.
// A causal mask is computed from the indices; any other mask is packed into bits once per CTA.
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

__device__ __forceinline__ float4 lo4(const float4& x) { return make_float4(tf32_lo(x.x), tf32_lo(x.y), tf32_lo(x.z), tf32_lo(x.w)); }

// The transpose of a 128-row global block of C columns (C = 32 or 64): source rows become the
// tile's K index and source columns its rows (a K-major tile of C rows over K = 128). Thread i
// takes the 4 x 4 block i (source rows j..j+3, columns e..e+3); blockDim.x >= 8 C, so one block
// per thread. Split into the loads (issued early, before a wait) and the transposed stores.
struct TBlock {
  float4 x[4];
  int e, j;
  bool on;
};
__device__ __forceinline__ TBlock load_t(const float* __restrict__ src, int C, long long ld) {
  TBlock b;
  const int c4 = C >> 2, i = threadIdx.x;
  b.on = i < 32 * c4;
  const int jb = i / c4;
  b.e = (i - jb * c4) << 2;
  b.j = jb << 2;
  if (b.on) {
#pragma unroll
    for (int u = 0; u < 4; ++u) b.x[u] = *(const float4*)(src + (long long)(b.j + u) * ld + b.e);
  }
  return b;
}
__device__ __forceinline__ void store_t(uint8_t* hi, uint8_t* lo, const TBlock& b, int C) {
  if (!b.on) return;
  const float4 t[4] = {make_float4(b.x[0].x, b.x[1].x, b.x[2].x, b.x[3].x), make_float4(b.x[0].y, b.x[1].y, b.x[2].y, b.x[3].y),
                       make_float4(b.x[0].z, b.x[1].z, b.x[2].z, b.x[3].z), make_float4(b.x[0].w, b.x[1].w, b.x[2].w, b.x[3].w)};
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint32_t off = kmaj(C, b.e + u, b.j);
    *(float4*)(hi + off) = t[u];
    *(float4*)(lo + off) = lo4(t[u]);
  }
}

// Instruction descriptor: M x N, TF32 x TF32 -> F32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (128 x N) (+)= A (128 x K) B (N x K)^T in 3xTF32, A and B K-major hi/lo tiles (shared-memory
// addresses; B's tile has N rows). Issued by one thread, fully unrolled: the descriptors are
// formed once and stepped by constant offsets (the address field is address / 16).
template <int N, int K>
__device__ __forceinline__ void mma3(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl, uint32_t idesc, bool accumulate) {
  const uint64_t dah = desc_k(ah), dal = desc_k(al), dbh = desc_k(bh), dbl = desc_k(bl);
#pragma unroll
  for (int kb = 0; kb < K / 32; ++kb) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ao = (uint64_t)((kb * 128 * 128 + kk * 32) >> 4), bo = (uint64_t)((kb * N * 128 + kk * 32) >> 4);
      mma_tf32(d, dah + ao, dbh + bo, idesc, (accumulate || kb || kk) ? 1u : 0u);
      mma_tf32(d, dah + ao, dbl + bo, idesc, 1u);
      mma_tf32(d, dal + ao, dbh + bo, idesc, 1u);
    }
  }
}

// Two row-major blocks into K-major hi / lo tiles, each thread's loads (up to eight 16-byte
// vectors) issued before its stores: A with RA rows (row stride lda floats) and B with RB rows
// (row stride ldb), K columns each, 16-byte aligned rows.
__device__ __forceinline__ void stage2(uint8_t* ah, uint8_t* al, const float* __restrict__ a, int RA, long long lda, uint8_t* bh, uint8_t* bl,
                                       const float* __restrict__ b, int RB, long long ldb, int K) {
  const int k4 = K >> 2, na = RA * k4, n = na + RB * k4, step = blockDim.x;
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * step) {
    float4 x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * step;
      if (i < n) {
        const bool in_a = i < na;
        const int e = in_a ? i : i - na, row = e / k4, col = (e - row * k4) << 2;
        x[u] = *(const float4*)(in_a ? a + row * lda + col : b + row * ldb + col);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * step;
      if (i < n) {
        const bool in_a = i < na;
        const int e = in_a ? i : i - na, row = e / k4, col = (e - row * k4) << 2;
        const uint32_t off = kmaj(in_a ? RA : RB, row, col);
        *(float4*)((in_a ? ah : bh) + off) = x[u];
        *(float4*)((in_a ? al : bl) + off) = lo4(x[u]);
      }
    }
  }
}

// stage2 split in two, with all of a thread's vectors (U of them; U blockDim.x >= the block's
// vector count) loaded at once, so that the loads can be issued before other work and the
// stores made later.
template <int U> struct Staged {
  float4 x[U];
};
template <int U>
__device__ __forceinline__ void load2(Staged<U>& st, const float* __restrict__ a, int RA, long long lda, const float* __restrict__ b, int RB,
                                      long long ldb, int K) {
  const int k4 = K >> 2, na = RA * k4, n = na + RB * k4;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
    if (i < n) {
      const bool in_a = i < na;
      const int e = in_a ? i : i - na, row = e / k4, col = (e - row * k4) << 2;
      st.x[u] = *(const float4*)(in_a ? a + row * lda + col : b + row * ldb + col);
    }
  }
}
template <int U>
__device__ __forceinline__ void store2(const Staged<U>& st, uint8_t* ah, uint8_t* al, int RA, uint8_t* bh, uint8_t* bl, int RB, int K) {
  const int k4 = K >> 2, na = RA * k4, n = na + RB * k4;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int i = threadIdx.x + u * blockDim.x;
    if (i < n) {
      const bool in_a = i < na;
      const int e = in_a ? i : i - na, row = e / k4, col = (e - row * k4) << 2;
      const uint32_t off = kmaj(in_a ? RA : RB, row, col);
      *(float4*)((in_a ? ah : bh) + off) = st.x[u];
      *(float4*)((in_a ? al : bl) + off) = lo4(st.x[u]);
    }
  }
}

// TMEM stores of 16 or 32 consecutive columns of the warp's 32 lanes; tmem_st_wait makes them
// complete before the fence and barrier that hand them to a product.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
      "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]),
      "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,"
      "%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
      "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One TF32 product with A (128 rows = TMEM lanes, 8 K columns from column address `a`) in TMEM
// and B from shared memory.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  const uint32_t no_mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}

// D (128 x N) (+)= A (128 x K) B (N x K)^T in 3xTF32 with A in TMEM: hi in columns ah .. ah + K - 1,
// lo in al .. al + K - 1 (row = lane); B a K-major hi / lo tile pair in shared memory (N rows).
// Fully unrolled, descriptors stepped by constant offsets as in mma3.
template <int N, int K>
__device__ __forceinline__ void mma3_ts(uint32_t d, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl, uint32_t idesc, bool accumulate) {
  const uint64_t dbh = desc_k(bh), dbl = desc_k(bl);
#pragma unroll
  for (int kb = 0; kb < K / 32; ++kb) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t ao = (uint32_t)(kb * 32 + kk * 8);
      const uint64_t bo = (uint64_t)((kb * N * 128 + kk * 32) >> 4);
      mma_tf32_ts(d, ah + ao, dbh + bo, idesc, (accumulate || kb || kk) ? 1u : 0u);
      mma_tf32_ts(d, ah + ao, dbl + bo, idesc, 1u);
      mma_tf32_ts(d, al + ao, dbh + bo, idesc, 1u);
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

// Bounded wait on `bar` for its next phase; `count` tracks the phases already consumed.
__device__ __forceinline__ bool cta_next(uint64_t* bar, int& count, volatile int* abort, int* err, int code) {
  const bool ok = cta_wait(bar, (uint32_t)(count & 1), abort, err, code);
  ++count;
  return ok;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]),
        "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
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

// ---------------------------------------------------------------------------------------------
// Mask bits
// ---------------------------------------------------------------------------------------------
// A causal mask (mask[i][j] != 0 exactly where j <= i: a constant lower triangle, recognised by
// the planner) is computed from the indices and never read. Any other mask is packed once per
// CTA into words in shared memory, bit (j - j0) % 32 of words[(i - i0) * (C / 32) + (j - j0) / 32]
// set where mask[i][j] != 0, for rows [i0, i0 + R) and columns [j0, j0 + C) (C a multiple of
// 32): one coalesced 128-byte load and one ballot per word, eight loads in flight per warp.

// Keys j0 .. j0 + 31 of query i under the causal mask.
__device__ __forceinline__ uint32_t causal_keys(int i, int j0) {
  const int n = i - j0 + 1;
  return n <= 0 ? 0u : n >= 32 ? 0xffffffffu : ((1u << n) - 1u);
}
// Queries i0 .. i0 + 31 of key j under the causal mask.
__device__ __forceinline__ uint32_t causal_queries(int j, int i0) {
  const int n = j - i0;
  return n <= 0 ? 0xffffffffu : n >= 32 ? 0u : (0xffffffffu << n);
}

__device__ void pack_mask(uint32_t* words, const float* __restrict__ mask, int T, int i0, int R, int j0, int C) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int wpr = C >> 5, n = R * wpr;
  for (int b = warp; b < n; b += 8 * nw) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int it = b + u * nw;
      x[u] = 0.0f;
      if (it < n) {
        const int row = it / wpr, w = it - row * wpr;
        x[u] = mask[(long long)(i0 + row) * T + j0 + 32 * w + lane];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int it = b + u * nw;
      const uint32_t bits = __ballot_sync(FULL, x[u] != 0.0f);
      if (lane == 0 && it < n) words[it] = bits;
    }
  }
}

// Per query row of a 128-row block (global rows row0 ..): the forward's row maximum m and
// 1 / exp-sum, and D = rowsum(dO * O) with O read from the forward's packed output. Warp w
// takes rows 8 w .. 8 w + 7, lanes over the row's columns; st[0..127] = m, st[128..255] = 1 / s,
// st[256..383] = D.
template <int D>
__device__ __forceinline__ void query_stats(float* st, const float* __restrict__ fwd, const float* __restrict__ dout, long long ldo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int PER = D / 32;
  float a[8][PER], o[8][PER], ms[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const long long r = warp * 8 + u;
#pragma unroll
    for (int p = 0; p < PER; ++p) {
      a[u][p] = dout[r * ldo + p * 32 + lane];
      o[u][p] = fwd[r * (D + 2) + p * 32 + lane];
    }
    ms[u] = lane < 2 ? fwd[r * (D + 2) + D + lane] : 0.0f;  // lane 0: m, lane 1: s
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    float s = a[u][0] * o[u][0];
#pragma unroll
    for (int p = 1; p < PER; ++p) s = s + a[u][p] * o[u][p];
#pragma unroll
    for (int off = 16; off; off >>= 1) s = s + __shfl_xor_sync(FULL, s, off);
    const float mu = __shfl_sync(FULL, ms[u], 0), su = __shfl_sync(FULL, ms[u], 1);
    const int rl = warp * 8 + u;
    if (lane == 0) {
      st[rl] = mu;
      st[128 + rl] = 1.0f / su;
      st[256 + rl] = s;
    }
  }
}

constexpr int FWD_THREADS = 512;

// Where batch entry z's rows live (AttnShape::heads): with heads = 0, q, k, v and dO are (Z, T, d)
// row blocks and the backward writes (Z, T, 3 d) rows; with heads = H > 0, entry z = b H + h of
// q, k, v is part 0, 1, 2 of the packed (B, T, 3, H, d) tensor (row stride 3 H d), dO is
// (B, T, H, d) (row stride H d) and the backward writes the packed tensor's gradient.
template <int T, int D> struct Rows {
  long long xo, ld, dO, ldo;  // q / k / v offset of row 0 and row stride; the same for dO
  int heads;
  long long z;
  __device__ Rows(long long z_, int heads_) : heads(heads_), z(z_) {
    if (heads) {
      const long long b = z / heads, h = z - b * heads;
      xo = (b * T * 3 * heads + h) * D;
      ld = 3LL * heads * D;
      dO = (b * T * heads + h) * D;
      ldo = (long long)heads * D;
    } else {
      xo = dO = z * T * D;
      ld = ldo = D;
    }
  }
  // Offset of part w (0 dq, 1 dk, 2 dv) of row t in the backward's result.
  __device__ long long grad(int t, int w) const { return heads ? xo + t * ld + (long long)w * heads * D : (z * T + t) * 3 * D + (long long)w * D; }
};

template <int T, int D> struct FwdLayout {
  static constexpr int QB = 128 * D * 4, KB = T * D * 4;
  static constexpr int VB = D * 128 * 4;  // v^T of one half of the keys: D rows over 128 keys
  static constexpr int PHASE1 = 2 * QB + 2 * KB, PHASE2 = 2 * VB * (T / 128);
  static constexpr int REGION = PHASE1 > PHASE2 ? PHASE1 : PHASE2;
  static constexpr int WORDS = 128 * (T / 32) * 4;  // the mask bits of the block's rows
  static constexpr int SMEM = 1024 + REGION + WORDS + 2 * 4 * 128 * 4 + 128;
  static constexpr uint32_t LO = T + D;  // TMEM: S (and E) [0, T), O [T, T + D), E lo [LO, LO + 128)
  static_assert(LO + 128 <= 512, "TMEM columns");
  static_assert(128 * (D + 2) * 4 <= REGION, "output staging fits the operand region");
};

// Forward, one CTA of 16 warps per (batch entry, 128 query rows). Warp w reads TMEM lanes
// 32 (w % 4) .. +31 (query rows) and, as group g = w / 4, the key chunk g of every half of
// 128 keys, so the four warps of a row share its 32-column chunks. S = q k^T lands in TMEM;
// v^T of both halves is staged once the product is done (the loads in flight across its
// wait). Pass 1 gives each row's maximum (partial maxima combined through shared memory).
// Per half of the keys, E = exp(Z - m) replaces the half's S columns in TMEM (the hi part) and
// its lo part goes to a TMEM buffer; O += E v takes E from TMEM. O is divided by the row's
// exp-sum and the block's packed rows (O, m, s) leave through shared memory as one
// contiguous, coalesced store.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_fwd_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                              const float* __restrict__ v, const float* __restrict__ mask, int causal, int heads,
                                                              float inv_c, float fill, int* err) {
  using L = FwdLayout<T, D>;
  constexpr int NQB = T / 128, NH = T / 128, NW = T / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Qh = sm, *Ql = Qh + L::QB, *Kh = Ql + L::QB, *Kl = Kh + L::KB;  // phase 1
  uint8_t* V0 = sm;                                                         // phase 2: half h at V0 + 2 h VB (hi), + VB (lo)
  float* ost = (float*)sm;                                                  // epilogue: the block's packed rows
  uint32_t* words = (uint32_t*)(sm + L::REGION);                            // [128][NW]
  float* part = (float*)(sm + L::REGION + L::WORDS);                        // [2][4][128]: partial max, partial sum
  uint64_t* bars = (uint64_t*)(part + 2 * 4 * 128);
  uint64_t *bar_s = bars, *bar_o = bars + 1, *bar_done = bars + 2;
  uint32_t* tslot = (uint32_t*)(bars + 3);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;  // this thread's query row within the block
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + row;
  const Rows<T, D> rows(z, heads);
  q += rows.xo + r0 * rows.ld;
  k += rows.xo;
  v += rows.xo;
  // q and k in flight across the set-up (all of a thread's vectors at once).
  constexpr int UQK = ((128 + T) * D / 4 + FWD_THREADS - 1) / FWD_THREADS;
  Staged<UQK> qk;
  load2(qk, q, 128, rows.ld, k, T, rows.ld, D);

  if (tid == 0) {
    for (int b = 0; b < 3; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(512u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (!causal) pack_mask(words, mask, T, r0, 128, 0, T);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lanes = (uint32_t)(lq * 32) << 16;
  const uint32_t S_t = tmem, O_t = tmem + T, LO_t = tmem + L::LO;

  // S = q k^T.
  store2(qk, Qh, Ql, 128, Kh, Kl, T, D);
  proxy_fence();
  __syncthreads();
  if (tid == 0) {
    fence_after();
    mma3<T, D>(S_t, saddr(Qh), saddr(Ql), saddr(Kh), saddr(Kl), idesc_tf32(128, T), false);
    mma_commit(bar_s);
  }
  TBlock vb = load_t(v, D, rows.ld);  // v^T of the first half, in flight across the wait
  bool ok = cta_wait(bar_s, 0, abort, err, 21);
  fence_after();
  store_t(V0, V0 + L::VB, vb, D);
  if (NH > 1) vb = load_t(v + 128 * rows.ld, D, rows.ld);

  // Pass 1: the mask bits of this thread's chunks and the row maximum.
  uint32_t bits[NH];
  float m = -INFINITY;
  if (ok) {
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      const int c0 = h * 128 + g * 32;
      uint32_t x[32];
      tmem_ld32(S_t + lanes + c0, x);
      const uint32_t b = causal ? causal_keys(r, c0) : words[row * NW + (c0 >> 5)];
      bits[h] = b;
#pragma unroll
      for (int j = 0; j < 32; ++j) m = nan_max(m, ((b >> j) & 1u) ? __uint_as_float(x[j]) * inv_c : fill);
    }
    part[g * 128 + row] = m;
  }
  if (NH > 1) store_t(V0 + 2 * L::VB, V0 + 3 * L::VB, vb, D);
  __syncthreads();
  if (ok) m = nan_max(nan_max(part[row], part[128 + row]), nan_max(part[256 + row], part[384 + row]));

  // Per half of the keys: E over the half's S columns (hi) and into the lo buffer, then O += E v.
  float sum = 0.0f;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    const int c0 = h * 128 + g * 32;
    uint32_t x[32];
    tmem_ld32(S_t + lanes + c0, x);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float e = __expf((((bits[h] >> j) & 1u) ? __uint_as_float(x[j]) * inv_c : fill) - m);
      sum = sum + e;
      x[j] = __float_as_uint(e);
    }
    tmem_st32(S_t + lanes + c0, x);
    // The lo buffer is free once the previous half's products are done.
    if (h > 0 && !(ok = cta_wait(bar_o, (uint32_t)((h - 1) & 1), abort, err, 22))) break;
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __float_as_uint(tf32_lo(__uint_as_float(x[j])));
    tmem_st32(LO_t + lanes + g * 32, x);
    tmem_st_wait();
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      uint8_t* vh = V0 + 2 * h * L::VB;
      mma3_ts<D, 128>(O_t, S_t + h * 128, LO_t, saddr(vh), saddr(vh + L::VB), idesc_tf32(128, D), h > 0);
      mma_commit(bar_o);
    }
  }
  if (ok) ok = cta_wait(bar_o, (uint32_t)((NH - 1) & 1), abort, err, 23);
  fence_after();
  if (ok) part[512 + g * 128 + row] = sum;
  __syncthreads();

  // O / s, m and s of row `row` into the staging rows (group g: O columns [32 g, 32 g + 32)),
  // then the block's 128 (D + 2)-float rows, contiguous in `out`, in 16-byte stores.
  if (ok) {
    const float s4 = (part[512 + row] + part[640 + row]) + (part[768 + row] + part[896 + row]);
    float* orow = ost + row * (D + 2);
    if (g * 32 < D) {
      uint32_t x[32];
      tmem_ld32(O_t + lanes + g * 32, x);
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *(float2*)(orow + g * 32 + j) = make_float2(__uint_as_float(x[j]) / s4, __uint_as_float(x[j + 1]) / s4);
    }
    if (g == 0) *(float2*)(orow + D) = make_float2(m, s4);
  }
  __syncthreads();
  if (ok) {
    float4* dst = (float4*)(out + (z * T + r0) * (D + 2));
    const float4* srcv = (const float4*)ost;
    for (int i = tid; i < 32 * (D + 2); i += FWD_THREADS) dst[i] = srcv[i];
  }
  tc_teardown(bar_done, tmem, 512u);
}

// Shared-memory plan of the backward kernels: region 0 stages two 128-row operands (hi and lo)
// for the score products; region 1 one transposed operand (D rows over 128 columns, hi and lo);
// then the query statistics and the mask words. TMEM: the scores (then P or its transpose, hi)
// [0, 128), dP (then dS, hi) [128, 256), a lo buffer of 128 columns and the accumulators.
template <int T, int D> struct BwdLayout {
  static constexpr int TB = 128 * D * 4;  // a 128 x D tile, or its transpose
  static constexpr int R0 = 4 * TB, R1 = 2 * TB;
  static constexpr int REGION = R0 + R1;
  static constexpr int WORDS = 128 * (T / 32) * 4;
  static constexpr int SMEM = 1024 + REGION + 3 * 128 * 4 + WORDS + 128;
  static_assert(128 * (2 * D + 4) * 4 <= REGION, "output staging fits the operand region");
  static_assert(384 + 2 * D <= 512, "TMEM columns");
};

// dq, one CTA of 16 warps per (batch entry, 128 query rows); warp w reads TMEM lanes 32 (w % 4)
// (query rows) and, as group g = w / 4, key chunk g of each half. Per half of the keys (128):
// S = q k^T, then dP = dO v^T with k^T of the half staged beside it; dS replaces S in TMEM (hi)
// with its lo part in the lo buffer, and dq += dS k takes dS from TMEM. dq leaves through
// shared memory in row-contiguous stores.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_dq_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                             const float* __restrict__ v, const float* __restrict__ mask, const float* __restrict__ fwd,
                                                             const float* __restrict__ dout, float* __restrict__ qstats, int causal, int heads,
                                                             float inv_c, float fill, int* err) {
  using L = BwdLayout<T, D>;
  constexpr int NQB = T / 128, NH = T / 128, NW = T / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // region 0
  uint8_t *Xh = sm + L::R0, *Xl = Xh + L::TB;                            // region 1: k^T of the half
  float* stats = (float*)(sm + L::REGION);                                // [3][128]
  uint32_t* words = (uint32_t*)(stats + 3 * 128);                         // [128][NW]
  uint64_t* bars = (uint64_t*)(sm + L::REGION + 3 * 128 * 4 + L::WORDS);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_done = bars + 3;
  uint32_t* tslot = (uint32_t*)(bars + 4);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;
  const long long z = blockIdx.x / NQB;
  const int r0 = (int)(blockIdx.x - z * NQB) * 128, r = r0 + row;
  const Rows<T, D> rows(z, heads);
  const long long ld = rows.ld, ldo = rows.ldo;
  const float* qb = q + rows.xo + r0 * ld;
  const float* db = dout + rows.dO + r0 * ldo;
  k += rows.xo;
  v += rows.xo;

  if (tid == 0) {
    for (int b = 0; b < 4; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(512u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  query_stats<D>(stats, fwd + (z * T + r0) * (D + 2), db, ldo);
  if (!causal) pack_mask(words, mask, T, r0, 128, 0, T);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot, lanes = (uint32_t)(lq * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, Q_t = tmem + 256, LO_t = tmem + 256 + D;
  const float m = stats[row], inv_sum = stats[128 + row], Dr = stats[256 + row];
  // The block's query statistics for the dk / dv kernel: m, 1 / s and D, each a (Z, T) array.
  if (tid < 128) {
    const long long zt = (long long)(gridDim.x / NQB) * T, at = z * T + r0 + tid;
    qstats[at] = stats[tid];
    qstats[zt + at] = stats[128 + tid];
    qstats[2 * zt + at] = stats[256 + tid];
  }

  bool ok = true;
  int na = 0, nb = 0, nc = 0;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    // a: S = q k_h^T (the previous half's products are complete).
    stage2(Ah, Al, qb, 128, ld, Bh, Bl, k + h * 128 * ld, 128, ld, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3<128, D>(S_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), idesc_tf32(128, 128), false);
      mma_commit(bar_a);
    }
    const TBlock kt = load_t(k + h * 128 * ld, D, ld);
    if (!(ok = cta_next(bar_a, na, abort, err, 31))) break;
    // b: dP = dO v_h^T, and k_h^T in region 1.
    stage2(Ah, Al, db, 128, ldo, Bh, Bl, v + h * 128 * ld, 128, ld, D);
    store_t(Xh, Xl, kt, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3<128, D>(P_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), idesc_tf32(128, 128), false);
      mma_commit(bar_b);
    }
    if (!(ok = cta_next(bar_b, nb, abort, err, 32))) break;
    fence_after();
    // c: this group's dS chunk in two 16-column pieces, hi over S and lo into the buffer.
    {
      const int c0 = h * 128 + g * 32;
      const uint32_t bits = causal ? causal_keys(r, c0) : words[row * NW + (c0 >> 5)];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        uint32_t xs[16], xp[16];
        tmem_ld16(S_t + lanes + g * 32 + 16 * p, xs);
        tmem_ld16(P_t + lanes + g * 32 + 16 * p, xp);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool on = (bits >> (16 * p + j)) & 1u;
          const float pr = __expf((on ? __uint_as_float(xs[j]) * inv_c : fill) - m) * inv_sum;
          const float ds = on ? pr * (__uint_as_float(xp[j]) - Dr) * inv_c : 0.0f;
          xs[j] = __float_as_uint(ds);
          xp[j] = __float_as_uint(tf32_lo(ds));
        }
        tmem_st16(S_t + lanes + g * 32 + 16 * p, xs);
        tmem_st16(LO_t + lanes + g * 32 + 16 * p, xp);
      }
    }
    tmem_st_wait();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3_ts<D, 128>(Q_t, S_t, LO_t, saddr(Xh), saddr(Xl), idesc_tf32(128, D), h > 0);
      mma_commit(bar_c);
    }
    if (!(ok = cta_next(bar_c, nc, abort, err, 33))) break;
    fence_after();
  }
  // dq rows through shared memory (pitch D + 4 floats), then D-float row segments of `out`.
  float* ost = (float*)sm;
  if (ok && g * 32 < D) {
    uint32_t x[32];
    tmem_ld32(Q_t + lanes + g * 32, x);
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *(float4*)(ost + row * (D + 4) + g * 32 + j) =
          make_float4(__uint_as_float(x[j]), __uint_as_float(x[j + 1]), __uint_as_float(x[j + 2]), __uint_as_float(x[j + 3]));
  }
  __syncthreads();
  if (ok) {
    constexpr int V4 = D / 4;  // 16-byte vectors per row
    for (int i = tid; i < 128 * V4; i += FWD_THREADS) {
      const int rr = i / V4, c = (i - rr * V4) * 4;
      *(float4*)(out + rows.grad(r0 + rr, 0) + c) = *(const float4*)(ost + rr * (D + 4) + c);
    }
  }
  tc_teardown(bar_done, tmem, 512u);
}

// dk and dv, one CTA of 16 warps per (batch entry, 128 keys); warp w reads TMEM lanes 32 (w % 4)
// (key rows) and, as group g = w / 4, query chunk g of each half. Per half of the queries
// (128): S^T = k q^T; dP^T = v dO^T with dO^T of the half staged beside it; P^T replaces S^T in
// TMEM (hi, lo in the buffer) and dv += P^T dO; then, with q^T staged over the score operands,
// dS^T replaces dP^T (hi, lo in the buffer) and dk += dS^T q. The half's query statistics (max,
// 1 / exp-sum, D), which the dq kernel leaves in `qstats`, sit in shared memory. dk and dv leave
// through shared memory.
template <int T, int D>
__global__ void __launch_bounds__(FWD_THREADS, 1) k_attn_dkdv_tc(float* __restrict__ out, const float* __restrict__ q, const float* __restrict__ k,
                                                               const float* __restrict__ v, const float* __restrict__ mask,
                                                               const float* __restrict__ fwd, const float* __restrict__ dout,
                                                               const float* __restrict__ qstats, int causal, int heads, float inv_c, float fill, int* err) {
  using L = BwdLayout<T, D>;
  constexpr int NKB = T / 128, NH = T / 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *Ah = sm, *Al = Ah + L::TB, *Bh = Al + L::TB, *Bl = Bh + L::TB;  // region 0; q^T of the half at Ah / Al after dP^T
  uint8_t *Xh = sm + L::R0, *Xl = Xh + L::TB;                            // region 1: dO^T of the half
  float* stats = (float*)(sm + L::REGION);                                // [3][128]
  uint32_t* words = (uint32_t*)(stats + 3 * 128);                         // [T][4]: queries x the block's 128 keys
  uint64_t* bars = (uint64_t*)(sm + L::REGION + 3 * 128 * 4 + L::WORDS);
  uint64_t *bar_a = bars, *bar_b = bars + 1, *bar_c = bars + 2, *bar_d = bars + 3, *bar_done = bars + 4;
  uint32_t* tslot = (uint32_t*)(bars + 5);
  volatile int* abort = (volatile int*)(tslot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, lq = warp & 3, g = warp >> 2;
  const int row = lq * 32 + lane;  // key row within the block
  const long long z = blockIdx.x / NKB;
  const int j0 = (int)(blockIdx.x - z * NKB) * 128, j = j0 + row;
  const Rows<T, D> rows(z, heads);
  const long long ld = rows.ld, ldo = rows.ldo;
  const float* kb = k + rows.xo + j0 * ld;
  const float* vb = v + rows.xo + j0 * ld;
  const float* qz = q + rows.xo;
  const float* dz = dout + rows.dO;

  if (tid == 0) {
    for (int b = 0; b < 5; ++b) mbar_init(&bars[b], 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tslot)), "r"(512u) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (!causal) pack_mask(words, mask, T, 0, T, j0, 128);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tslot, lanes = (uint32_t)(lq * 32) << 16;
  const uint32_t S_t = tmem, P_t = tmem + 128, LO_t = tmem + 256, V_t = tmem + 384, K_t = tmem + 384 + D;

  bool ok = true;
  int na = 0, nb = 0, nc = 0, nd = 0;
#pragma unroll 1
  for (int h = 0; h < NH && ok; ++h) {
    const int q0 = h * 128;
    // The half's query statistics, from the dq kernel (the previous half's readers finished at
    // its last wait).
    if (tid < 128) {
      const long long zt = (long long)(gridDim.x / NKB) * T, at = z * T + q0 + tid;
      stats[tid] = qstats[at];
      stats[128 + tid] = qstats[zt + at];
      stats[256 + tid] = qstats[2 * zt + at];
    }
    // a: S^T = k q_h^T.
    stage2(Ah, Al, kb, 128, ld, Bh, Bl, qz + q0 * ld, 128, ld, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3<128, D>(S_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), idesc_tf32(128, 128), false);
      mma_commit(bar_a);
    }
    const TBlock dt = load_t(dz + q0 * ldo, D, ldo);
    // The mask bits of this key over the chunk's queries q0 + 32 g ...
    uint32_t qbits = 0;
    if (causal) {
      qbits = causal_queries(j, q0 + g * 32);
    } else {
#pragma unroll 8
      for (int i = 0; i < 32; ++i) qbits |= ((words[(q0 + g * 32 + i) * 4 + (row >> 5)] >> lane) & 1u) << i;
    }
    if (!(ok = cta_next(bar_a, na, abort, err, 41))) break;
    // b: dP^T = v dO_h^T, and dO_h^T in region 1.
    stage2(Ah, Al, vb, 128, ld, Bh, Bl, dz + q0 * ldo, 128, ldo, D);
    store_t(Xh, Xl, dt, D);
    proxy_fence();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3<128, D>(P_t, saddr(Ah), saddr(Al), saddr(Bh), saddr(Bl), idesc_tf32(128, 128), false);
      mma_commit(bar_b);
    }
    fence_after();
    // c1: this group's P^T chunk (query columns q0 + 32 g ..) over S^T (hi) and into the buffer.
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint32_t xs[16], xl[16];
      tmem_ld16(S_t + lanes + g * 32 + 16 * p, xs);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rl = g * 32 + 16 * p + i;
        const float pv = __expf((((qbits >> (16 * p + i)) & 1u) ? __uint_as_float(xs[i]) * inv_c : fill) - stats[rl]) * stats[128 + rl];
        xs[i] = __float_as_uint(pv);
        xl[i] = __float_as_uint(tf32_lo(pv));
      }
      tmem_st16(S_t + lanes + g * 32 + 16 * p, xs);
      tmem_st16(LO_t + lanes + g * 32 + 16 * p, xl);
    }
    tmem_st_wait();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3_ts<D, 128>(V_t, S_t, LO_t, saddr(Xh), saddr(Xl), idesc_tf32(128, D), h > 0);
      mma_commit(bar_c);
    }
    const TBlock qt = load_t(qz + q0 * ld, D, ld);
    // dP^T done: region 0 takes q_h^T. dv done: the lo buffer is free.
    if (!(ok = cta_next(bar_b, nb, abort, err, 42))) break;
    store_t(Ah, Al, qt, D);
    if (!(ok = cta_next(bar_c, nc, abort, err, 43))) break;
    fence_after();
    // c2: the dS^T chunk from P^T and dP^T in TMEM, over dP^T (hi) and into the buffer.
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      uint32_t xs[16], xp[16];
      tmem_ld16(S_t + lanes + g * 32 + 16 * p, xs);
      tmem_ld16(P_t + lanes + g * 32 + 16 * p, xp);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rl = g * 32 + 16 * p + i;
        const bool on = (qbits >> (16 * p + i)) & 1u;
        const float ds = on ? __uint_as_float(xs[i]) * (__uint_as_float(xp[i]) - stats[256 + rl]) * inv_c : 0.0f;
        xp[i] = __float_as_uint(ds);
        xs[i] = __float_as_uint(tf32_lo(ds));
      }
      tmem_st16(P_t + lanes + g * 32 + 16 * p, xp);
      tmem_st16(LO_t + lanes + g * 32 + 16 * p, xs);
    }
    tmem_st_wait();
    proxy_fence();
    fence_before();
    __syncthreads();
    if (tid == 0) {
      fence_after();
      mma3_ts<D, 128>(K_t, P_t, LO_t, saddr(Ah), saddr(Al), idesc_tf32(128, D), h > 0);
      mma_commit(bar_d);
    }
    if (!(ok = cta_next(bar_d, nd, abort, err, 44))) break;
    fence_after();
  }
  // dk and dv rows through shared memory (pitch 2 D + 4 floats), then 2 D-float row segments.
  float* ost = (float*)sm;
  if (ok && g * 32 < D) {
    uint32_t x[32];
    tmem_ld32(K_t + lanes + g * 32, x);
#pragma unroll
    for (int u = 0; u < 32; u += 4)
      *(float4*)(ost + row * (2 * D + 4) + g * 32 + u) =
          make_float4(__uint_as_float(x[u]), __uint_as_float(x[u + 1]), __uint_as_float(x[u + 2]), __uint_as_float(x[u + 3]));
    tmem_ld32(V_t + lanes + g * 32, x);
#pragma unroll
    for (int u = 0; u < 32; u += 4)
      *(float4*)(ost + row * (2 * D + 4) + D + g * 32 + u) =
          make_float4(__uint_as_float(x[u]), __uint_as_float(x[u + 1]), __uint_as_float(x[u + 2]), __uint_as_float(x[u + 3]));
  }
  __syncthreads();
  if (ok) {
    constexpr int V4 = D / 4;  // 16-byte vectors per row and part
    for (int i = tid; i < 128 * 2 * V4; i += FWD_THREADS) {
      const int rr = i / (2 * V4), rem = i - rr * 2 * V4, w = rem / V4, c = (rem - w * V4) * 4;
      *(float4*)(out + rows.grad(j0 + rr, 1 + w) + c) = *(const float4*)(ost + rr * (2 * D + 4) + w * D + c);
    }
  }
  tc_teardown(bar_done, tmem, 512u);
}

template <int T, int D> void set_smem() {
  cudaFuncSetAttribute(k_attn_fwd_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdLayout<T, D>::SMEM);
}

template <int T, int D> void launch_fwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const AttnShape& a, int* err,
                                           cudaStream_t s) {
  const long long blocks = a.batch * (T / 128);
  k_attn_fwd_tc<T, D><<<(unsigned)blocks, FWD_THREADS, FwdLayout<T, D>::SMEM, s>>>(out, q, k, v, mask, a.causal ? 1 : 0, a.heads, 1.0f / a.c, a.fill,
                                                                                  err);
}

template <int T, int D> void set_smem_bwd() {
  cudaFuncSetAttribute(k_attn_dq_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<T, D>::SMEM);
  cudaFuncSetAttribute(k_attn_dkdv_tc<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdLayout<T, D>::SMEM);
}

template <int T, int D> void launch_bwd_tc(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd,
                                           const float* dout, const AttnShape& a, float* qstats, int* err, cudaStream_t s) {
  const unsigned blocks = (unsigned)(a.batch * (T / 128));
  const int causal = a.causal ? 1 : 0;
  k_attn_dq_tc<T, D><<<blocks, FWD_THREADS, BwdLayout<T, D>::SMEM, s>>>(out, q, k, v, mask, fwd, dout, qstats, causal, a.heads, 1.0f / a.c, a.fill,
                                                                        err);
  k_attn_dkdv_tc<T, D><<<blocks, FWD_THREADS, BwdLayout<T, D>::SMEM, s>>>(out, q, k, v, mask, fwd, dout, qstats, causal, a.heads, 1.0f / a.c,
                                                                          a.fill, err);
}

}  // namespace

void attention_init() {
  static std::once_flag once;
  std::call_once(once, [] {
    set_smem<128, 32>();
    set_smem<128, 64>();
    set_smem<256, 32>();
    set_smem<256, 64>();
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
  if (a.heads) throw std::runtime_error("attention: the packed layout runs on the tensor-core kernels only");
  const long long rows = a.batch * a.t;
  k_attn_fwd_simt<<<(unsigned)((rows + 3) / 4), 128, 4 * a.t * sizeof(float), s>>>(out, q, k, v, mask, rows, a.t, a.d, a.dv, a.c, a.fill);
}

size_t attention_bwd_scratch_bytes(const AttnShape& a) { return attention_tc_supported(a) ? 3 * (size_t)a.batch * a.t * sizeof(float) : 0; }

void attention_bwd(float* out, const float* q, const float* k, const float* v, const float* mask, const float* fwd, const float* dout,
                   const AttnShape& a, void* scratch, int* error, cudaStream_t s) {
  if (a.batch == 0) return;
  if (attention_tc_supported(a)) {
    float* st = (float*)scratch;
    if (a.t == 128 && a.d == 32) return launch_bwd_tc<128, 32>(out, q, k, v, mask, fwd, dout, a, st, error, s);
    if (a.t == 128) return launch_bwd_tc<128, 64>(out, q, k, v, mask, fwd, dout, a, st, error, s);
    if (a.d == 32) return launch_bwd_tc<256, 32>(out, q, k, v, mask, fwd, dout, a, st, error, s);
    return launch_bwd_tc<256, 64>(out, q, k, v, mask, fwd, dout, a, st, error, s);
  }
  if (a.heads) throw std::runtime_error("attention: the packed layout runs on the tensor-core kernels only");
  const long long rows = a.batch * a.t;
  const unsigned blocks = (unsigned)((rows + 3) / 4);
  k_attn_dq_simt<<<blocks, 128, 4 * a.t * sizeof(float), s>>>(out, q, k, v, mask, fwd, dout, rows, a.t, a.d, a.dv, a.c, a.fill);
  k_attn_dkdv_simt<<<blocks, 128, 8 * a.t * sizeof(float), s>>>(out, q, k, v, mask, fwd, dout, rows, a.t, a.d, a.dv, a.c, a.fill);
}

}  // namespace rgc
