// fp32-accurate GEMM on sm_100a tensor cores: 3xTF32 with tcgen05.mma, TMEM accumulators and a
// TMA-fed, mbarrier-synchronised shared-memory pipeline (no cluster multicast).
//
// Each fp32 operand x is split, inside the kernel, into hi = x with its low 13 mantissa bits
// dropped (the TF32 value the tensor cores read from the raw fp32 tile, so hi needs no copy) and
// lo = x - hi (exact); C = A_hi B_hi + A_hi B_lo + A_lo B_hi, accumulated in fp32 in TMEM. The
// dropped A_lo B_lo term and the TF32 truncation of lo leave a relative error near 1e-6, well
// inside the 1e-4 parity bound.
//
// Persistent kernel, one CTA per SM, 10 warps:
//   warp 0      TMA producer: raw fp32 tiles of A (128 x 32) and B (BN x 32) per stage, in the
//               operands' own memory order (K-major, or MN-major for transposed storage).
//   warp 1      MMA issuer: three tcgen05.mma per 8-deep K step, into one of two TMEM
//               accumulators (128 lanes x BN fp32 columns each), so that a tile's epilogue
//               overlaps the next tile's main loop.
//   warps 2-5   converters: lo tiles beside the raw tiles; a proxy fence makes the
//               generic-proxy stores visible to the tensor cores.
//   warps 6-9   epilogue: tcgen05.ld of the accumulator, 16-byte stores to C (or to a split-K
//               partial, summed afterwards in split order, so results stay deterministic).
// Work units are (output tile, K split) pairs handed out round-robin over the persistent CTAs.
// Every wait is bounded by a wall-clock limit; on expiry the kernel records an error code, lets
// its copies and products in flight finish, frees its TMEM and exits.
//
// Pair form (PAIR = true, clusters of two CTAs on two SMs): the pair computes a 256 x BN tile
// with tcgen05.mma.cta_group::2 issued by the even CTA. Each CTA loads and converts its own 128
// rows of A and its own BN/2 columns of B; the tensor cores of both SMs read both halves of B,
// so each SM's shared memory carries half the B traffic and conversion work of the single-CTA
// form, and each CTA's TMEM holds the accumulator of its 128 rows. The odd CTA's converters and
// epilogue arrive on the even CTA's barriers through cluster addresses; the even CTA's commits
// signal both CTAs' barriers (one commit per CTA; no multicast).
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "gemm_tc.cuh"
#include "tc_common.cuh"

namespace rgc {

namespace {

using namespace tc;

constexpr int BM = 128, BK = 32;
constexpr int THREADS = 320;
constexpr uint32_t A_BYTES = BM * BK * 4;  // 16 KB

template <int BN, bool PAIR = false> struct Shape {
  static constexpr int BROWS = PAIR ? BN / 2 : BN;  // B rows (N columns) this CTA loads
  static constexpr uint32_t B_BYTES = BROWS * BK * 4;
  static constexpr uint32_t RAW = A_BYTES + B_BYTES;  // raw tiles (read by the MMA as hi)
  static constexpr uint32_t STAGE = 2 * RAW;          // + lo tiles
  static constexpr int STAGES = (200 * 1024) / STAGE > 4 ? 4 : (200 * 1024) / STAGE;
  // Epilogue staging: one 32 x 33-word block per epilogue warp, after the barriers.
  static constexpr uint32_t EPI = 4 * 32 * 33 * 4;
  static constexpr uint32_t SMEM = 1024 + STAGES * STAGE + 256 + EPI;
};

__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst), "l"(map),
      "r"(saddr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// MN-major tile: 32-element (128 B) runs along M or N, one per K row; a TMA box of 32 K rows
// (4 KB) per 32 MN elements. For 32-bit operands the tensor cores read MN-major tiles only in
// the "128-byte swizzle with 32-byte atoms" layout (layout type 1; TMA's SWIZZLE_128B_ATOM_32B):
// 4-row atoms of 512 B. Leading byte offset = next 32 MN elements (4 KB), stride byte offset =
// next 4 K rows (512 B).
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)(4096 >> 4) << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;
  return d;
}

// ---- CTA pairs (clusters of two) ----
__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_total() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// The cluster address of the barrier at the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  const uint32_t no_mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, "
      "p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}
// Completion of the pair's products so far, signalled on the barrier at cluster address `caddr`.
__device__ __forceinline__ void mma_commit_pair(uint32_t caddr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(caddr) : "memory");
}

struct Work {
  long long M, N;
  int mt, nt, batch, splits;
  int num_kb, kb_per_split;
  int za, zb;         // 1 when the operand has its own matrix per batch entry, else 0
  float* C;           // output (splits == 1) or partials [splits][batch][M][N]
};

template <int BN, bool AMN, bool BMN, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    k_tc3(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mB, const Work w, int* err) {
  using S = Shape<BN, PAIR>;
  constexpr int STAGES = S::STAGES;
  constexpr int TM = PAIR ? 2 * BM : BM;  // output rows per work unit
  constexpr int PEERS = PAIR ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * S::STAGE);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long units = (long long)w.mt * w.nt * w.batch * w.splits;
  // This CTA's place: rank within its pair (0 issues the products), first unit and stride.
  const uint32_t rank = PAIR ? cta_rank() : 0;
  const long long first_unit = PAIR ? (long long)cluster_index() : (long long)blockIdx.x;
  const long long unit_stride = PAIR ? (long long)cluster_total() : (long long)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4 * PEERS);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * PEERS);
    }
    mbar_init(done, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)), "r"((uint32_t)(2 * BN)) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)), "r"((uint32_t)(2 * BN)) : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  fence_before();
  __syncthreads();
  // Both CTAs' barriers exist before either arrives on the other's.
  if (PAIR) cluster_sync();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  auto decode = [&](long long u, int& m_t, int& n_t, int& z, int& sp) {
    n_t = (int)(u % w.nt);
    u /= w.nt;
    m_t = (int)(u % w.mt);
    u /= w.mt;
    z = (int)(u % w.batch);
    sp = (int)(u / w.batch);
  };
  auto kb_range = [&](int sp, int& kb0, int& kb1) {
    kb0 = sp * w.kb_per_split;
    kb1 = kb0 + w.kb_per_split < w.num_kb ? kb0 + w.kb_per_split : w.num_kb;
  };

  if (warp == 0) {
    if (lane == 0) {
      // Producer: this CTA's rows of A and columns of B.
      long long it = 0;
      for (long long u = first_unit; u < units && !*abort; u += unit_stride) {
        int m_t, n_t, z, sp, kb0, kb1;
        decode(u, m_t, n_t, z, sp);
        kb_range(sp, kb0, kb1);
        const int m0 = m_t * TM + (int)rank * BM, n0 = n_t * BN + (int)rank * S::BROWS;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          if (it >= STAGES && !mbar_wait(&empty[s], (uint32_t)(((it / STAGES) - 1) & 1), abort, err, 1)) break;
          mbar_expect_tx(&full[s], S::RAW);
          const uint32_t sa = saddr(smem + s * S::STAGE), sb = sa + A_BYTES;
          const int k0 = kb * BK;
          if (AMN) {
#pragma unroll
            for (int i = 0; i < BM / 32; ++i) tma_load(sa + i * 4096, &mA, &full[s], m0 + 32 * i, k0, z * w.za);
          } else {
            tma_load(sa, &mA, &full[s], k0, m0, z * w.za);
          }
          if (BMN) {
#pragma unroll
            for (int i = 0; i < S::BROWS / 32; ++i) tma_load(sb + i * 4096, &mB, &full[s], n0 + 32 * i, k0, z * w.zb);
          } else {
            tma_load(sb, &mB, &full[s], k0, n0, z * w.zb);
          }
        }
        if (*abort) break;
      }
      // Copies in flight land before the block's shared memory goes away.
      for (long long j = (it > STAGES ? it - STAGES : 0); j < it; ++j) {
        unsigned long long t0 = now_ns();
        while (!mbar_try(&full[j % STAGES], (uint32_t)((j / STAGES) & 1)) && now_ns() - t0 < WAIT_LIMIT_NS) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // MMA issuer. Instruction descriptor: M = TM, N = BN, TF32 x TF32 -> F32.
      const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((AMN ? 1u : 0u) << 15) | ((BMN ? 1u : 0u) << 16) |
                             ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
      long long it = 0, t = 0;
      for (long long u = first_unit; u < units && !*abort; u += unit_stride, ++t) {
        int m_t, n_t, z, sp, kb0, kb1;
        decode(u, m_t, n_t, z, sp);
        kb_range(sp, kb0, kb1);
        const int b = (int)(t & 1);
        if (t >= 2 && !mbar_wait<PAIR>(&acc_empty[b], (uint32_t)(((t >> 1) - 1) & 1), abort, err, 4)) break;
        fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        bool first = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = (int)(it % STAGES);
          if (!mbar_wait<PAIR>(&conv[s], (uint32_t)((it / STAGES) & 1), abort, err, 2)) break;
          fence_after();
          const uint32_t ah = saddr(smem + s * S::STAGE), bh = ah + A_BYTES;
          const uint32_t al = ah + S::RAW, bl = bh + S::RAW;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint32_t ka = AMN ? kk * 1024 : kk * 32, kb_ = BMN ? kk * 1024 : kk * 32;
            const uint64_t dah = AMN ? desc_mn(ah + ka) : desc_k(ah + ka), dal = AMN ? desc_mn(al + ka) : desc_k(al + ka);
            const uint64_t dbh = BMN ? desc_mn(bh + kb_) : desc_k(bh + kb_), dbl = BMN ? desc_mn(bl + kb_) : desc_k(bl + kb_);
            if (PAIR) {
              mma_tf32_pair(acc, dah, dbh, idesc, first ? 0u : 1u);
              mma_tf32_pair(acc, dah, dbl, idesc, 1);
              mma_tf32_pair(acc, dal, dbh, idesc, 1);
            } else {
              mma_tf32(acc, dah, dbh, idesc, first ? 0u : 1u);
              mma_tf32(acc, dah, dbl, idesc, 1);
              mma_tf32(acc, dal, dbh, idesc, 1);
            }
            first = false;
          }
          if (PAIR) {
            mma_commit_pair(cluster_addr(&empty[s], 0));
            mma_commit_pair(cluster_addr(&empty[s], 1));
          } else {
            mma_commit(&empty[s]);
          }
        }
        if (PAIR) {
          mma_commit_pair(cluster_addr(&acc_full[b], 0));
          mma_commit_pair(cluster_addr(&acc_full[b], 1));
        } else {
          mma_commit(&acc_full[b]);
        }
      }
      if (PAIR) {
        mma_commit_pair(cluster_addr(done, 0));
        mma_commit_pair(cluster_addr(done, 1));
      } else {
        mma_commit(done);
      }
    }
  } else if (warp < 6) {
    // Converters: 128 threads write each stage's lo tiles (the raw tiles serve as hi).
    const int ct = threadIdx.x - 64;
    long long it = 0;
    for (long long u = first_unit; u < units && !*abort; u += unit_stride) {
      int m_t, n_t, z, sp, kb0, kb1;
      decode(u, m_t, n_t, z, sp);
      kb_range(sp, kb0, kb1);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = (int)(it % STAGES);
        if (!mbar_wait(&full[s], (uint32_t)((it / STAGES) & 1), abort, err, 5)) {
          ok = false;
          break;
        }
        float4* raw = (float4*)(smem + s * S::STAGE);
        float4* lo = (float4*)(smem + s * S::STAGE + S::RAW);
#pragma unroll 4
        for (int i = ct; i < (int)(S::RAW / 16); i += 128) {
          const float4 v = raw[i];
          lo[i] = make_float4(v.x - tf32_trunc(v.x), v.y - tf32_trunc(v.y), v.z - tf32_trunc(v.z), v.w - tf32_trunc(v.w));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_remote(cluster_addr(&conv[s], 0));
          else mbar_arrive(&conv[s]);
        }
      }
      if (!ok) break;
    }
  } else {
    // Epilogue: warp w drains TMEM lanes [32 (w % 4), +32) = rows of this CTA's part of the tile.
    // For short K (at most 4 K blocks) the output dominates, and each 32 x 32 block goes through
    // shared memory (row pitch 33 words, conflict-free both ways) so that one warp store writes
    // four whole 128-byte row segments instead of 16 bytes in each of 32 rows. Longer K keeps the
    // direct stores: there the main loop is bound by shared-memory bandwidth.
    const int lg = warp & 3;
    const bool staged = w.num_kb <= 4;
    float* ep = (float*)(smem + STAGES * S::STAGE + 256) + lg * (32 * 33);
    const bool vec_out = (w.N % 4) == 0 && (((uintptr_t)w.C & 15) == 0);
    long long t = 0;
    for (long long u = first_unit; u < units && !*abort; u += unit_stride, ++t) {
      int m_t, n_t, z, sp;
      decode(u, m_t, n_t, z, sp);
      const int b = (int)(t & 1);
      if (!mbar_wait(&acc_full[b], (uint32_t)((t >> 1) & 1), abort, err, 3)) break;
      fence_after();
      const long long row = (long long)m_t * TM + (long long)rank * BM + lg * 32 + lane;
      const long long n0 = (long long)n_t * BN;
      float* out = w.C + (((long long)sp * w.batch + z) * w.M + row) * w.N;
      if (staged) {
        const long long row0 = row - lane;
        float* mat = w.C + ((long long)sp * w.batch + z) * w.M * w.N;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(b * BN + c), v);
#pragma unroll
          for (int j = 0; j < 32; ++j) ep[lane * 33 + j] = __uint_as_float(v[j]);
          __syncwarp();
          // Lane l stores columns 4 (l % 8) .. +3 of block row 4 i + l / 8.
          const long long col = n0 + c + (lane & 7) * 4;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = i * 4 + (lane >> 3);
            const float* src = ep + rr * 33 + (lane & 7) * 4;
            if (row0 + rr < w.M) {
              float* o = mat + (row0 + rr) * w.N + col;
              if (vec_out && col + 4 <= w.N) {
                *(float4*)o = make_float4(src[0], src[1], src[2], src[3]);
              } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  if (col + k < w.N) o[k] = src[k];
              }
            }
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(lg * 32) << 16) + (uint32_t)(b * BN + c), v);
        if (row < w.M) {
          float* o = out + n0 + c;
          const long long lim = w.N - (n0 + c);
          if (lim >= 32 && (((uintptr_t)o & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *(float4*)(o + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < lim) o[j] = __uint_as_float(v[j]);
          }
        }
      }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_remote(cluster_addr(&acc_empty[b], 0));
        else mbar_arrive(&acc_empty[b]);
      }
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0) {
    // Every product issued has completed before the accumulator is freed.
    unsigned long long t0 = now_ns();
    while (!mbar_try(done, 0) && now_ns() - t0 < WAIT_LIMIT_NS) {
    }
  }
  __syncthreads();
  // Neither CTA of a pair frees its TMEM or leaves (its shared memory holds operands and
  // barriers the other uses) before both are done.
  if (PAIR) cluster_sync();
  if (warp == 0) {
    fence_after();
    if (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN)) : "memory");
    else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * BN)) : "memory");
  }
}

// Split-K partials [splits][count] summed in split order.
__global__ void k_sum_splits(float* __restrict__ c, const float* __restrict__ part, long long count, int splits) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < count; e += (long long)gridDim.x * blockDim.x) {
    float acc = part[e];
    for (int s = 1; s < splits; ++s) acc = acc + part[(long long)s * count + e];
    c[e] = acc;
  }
}

// Copies rows x K operand matrices into K-major order with K padded to Kp (zeros), for operands
// whose own layout cannot be read by TMA (a row pitch that is not a multiple of 16 bytes).
// Element (z, r, k) is src[z * sz + r * K + k] (trans = false) or src[z * sz + k * R + r].
__global__ void k_pack(float* __restrict__ dst, const float* __restrict__ src, long long nmat, long long R, long long K, long long Kp, long long sz,
                       bool trans) {
  const long long n = nmat * R * Kp;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    long long k = e % Kp, rz = e / Kp, r = rz % R, z = rz / R;
    dst[e] = k < K ? src[z * sz + (trans ? k * R + r : r * K + k)] : 0.f;
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
#pragma GCC diagnostic push
#pragma GCC diagnostic ignored "-Wdeprecated-declarations"
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error("cuTensorMapEncodeTiled is not available");
#pragma GCC diagnostic pop
    return (EncodeTiled)p;
  }();
  return fn;
}

// A 3-D fp32 tensor map: dims {inner, outer, batch}, row stride and batch stride in elements.
CUtensorMap make_map(const float* base, long long inner, long long outer, long long batch, long long row_stride, long long batch_stride,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(row_stride * 4), (cuuint64_t)(std::max<long long>(batch_stride, row_stride * outer) * 4)};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (CUresult " + std::to_string((int)r) + ")");
  return m;
}

int pick_bn(long long n) { return n > 128 ? 256 : n > 64 ? 128 : 64; }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int sm_count() {
  static int sms = [] {
    int d = 0, v = 148;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    return v;
  }();
  return sms;
}

// Concurrently resident CTA pairs of the pair form (0 when pairs cannot be launched).
int g_pairs = 0;

// The launch decided for one product: operand layouts, packing, tile width, K splits.
struct Plan3 {
  bool pair;            // CTA-pair form (256-row tiles)
  bool a_mn, b_mn;      // operand read MN-major
  bool pack_a, pack_b;  // operand first packed K-major (row pitch not 16-byte aligned)
  long long kp;         // K of packed operands (multiple of 4)
  int bn, splits, num_kb, kb_per_split;
  long long mt, nt;
  size_t pack_a_bytes, pack_b_bytes, part_bytes;
};

Plan3 plan3(const TcGemm& g) {
  Plan3 p;
  // A is [m, k] (K-major) unless ta: [k, m] (MN-major). B is [k, n] (MN-major) unless tb: [n, k].
  p.a_mn = g.ta;
  p.b_mn = !g.tb;
  const long long pitch_a = p.a_mn ? g.m : g.k, pitch_b = p.b_mn ? g.n : g.k;
  p.pack_a = pitch_a % 4 != 0 || (g.batch_a % 4) != 0;
  p.pack_b = pitch_b % 4 != 0 || (g.batch_b % 4) != 0;
  p.kp = (g.k + 3) / 4 * 4;
  const long long nma = g.batch_a ? g.batch : 1, nmb = g.batch_b ? g.batch : 1;
  p.pack_a_bytes = p.pack_a ? align256((size_t)(nma * g.m * p.kp) * 4) : 0;
  p.pack_b_bytes = p.pack_b ? align256((size_t)(nmb * g.n * p.kp) * 4) : 0;
  if (p.pack_a) p.a_mn = false;
  if (p.pack_b) p.b_mn = false;
  p.bn = pick_bn(g.n);
  // Pairs of CTAs take 256-row tiles when there are rows for both and B is wide enough that
  // halving its per-SM traffic pays.
  p.pair = g_pairs > 0 && p.bn >= 128 && g.m > BM;
  const long long tm = p.pair ? 2 * BM : BM;
  p.mt = (g.m + tm - 1) / tm;
  p.nt = (g.n + p.bn - 1) / p.bn;
  p.num_kb = (int)((g.k + BK - 1) / BK);
  // Split K when the output tiles alone leave SMs idle: pick the split count (at least 8 K
  // blocks per split) that fills the most of whole waves, less a small charge per split for the
  // partial sums it writes and reads back.
  const long long tiles = p.mt * p.nt * g.batch, sms = p.pair ? g_pairs : sm_count();
  p.splits = 1;
  if (tiles < sms && p.num_kb >= 16) {
    double best = -1;
    for (int s = 1; s <= 32 && s * 8 <= p.num_kb; ++s) {
      long long units = tiles * s, waves = (units + sms - 1) / sms;
      double score = (double)units / (double)(waves * sms) - 0.003 * s;
      if (score > best + 1e-9) {
        best = score;
        p.splits = s;
      }
    }
  }
  p.kb_per_split = (p.num_kb + p.splits - 1) / p.splits;
  p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.part_bytes = p.splits > 1 ? align256((size_t)p.splits * (size_t)(g.batch * g.m * g.n) * 4) : 0;
  return p;
}

template <int BN, bool AMN, bool BMN, bool PAIR> void set_smem() {
  cudaError_t e = cudaFuncSetAttribute(k_tc3<BN, AMN, BMN, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Shape<BN, PAIR>::SMEM);
  if (e != cudaSuccess) throw std::runtime_error(std::string("tensor-core GEMM setup failed: ") + cudaGetErrorString(e));
}
template <int BN, bool PAIR> void set_smem_all() {
  set_smem<BN, false, false, PAIR>();
  set_smem<BN, false, true, PAIR>();
  set_smem<BN, true, false, PAIR>();
  set_smem<BN, true, true, PAIR>();
}

template <int BN, bool AMN, bool BMN, bool PAIR>
void launch_one(unsigned grid, const CUtensorMap& ma, const CUtensorMap& mb, const Work& w, int* err, cudaStream_t s) {
  const size_t smem = Shape<BN, PAIR>::SMEM;
  if constexpr (!PAIR) {
    k_tc3<BN, AMN, BMN, false><<<grid, THREADS, smem, s>>>(ma, mb, w, err);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_tc3<BN, AMN, BMN, true>, ma, mb, w, err);
    if (e != cudaSuccess) throw std::runtime_error(std::string("tensor-core GEMM launch failed: ") + cudaGetErrorString(e));
  }
}

template <int BN, bool PAIR>
void launch3(bool amn, bool bmn, unsigned grid, const CUtensorMap& ma, const CUtensorMap& mb, const Work& w, int* err, cudaStream_t s) {
  if (!amn && !bmn) launch_one<BN, false, false, PAIR>(grid, ma, mb, w, err, s);
  else if (!amn && bmn) launch_one<BN, false, true, PAIR>(grid, ma, mb, w, err, s);
  else if (amn && !bmn) launch_one<BN, true, false, PAIR>(grid, ma, mb, w, err, s);
  else launch_one<BN, true, true, PAIR>(grid, ma, mb, w, err, s);
}

// How many CTA pairs of the pair form can be resident at once (their shared memory puts one CTA
// on an SM; pairs must sit on two SMs of one cluster group).
template <int BN> int resident_pairs() {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * sm_count());
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = Shape<BN, true>::SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k_tc3<BN, false, false, true>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace

void tc_gemm_init() {
  static bool done = [] {
    set_smem_all<64, false>();
    set_smem_all<128, false>();
    set_smem_all<256, false>();
    set_smem_all<128, true>();
    set_smem_all<256, true>();
    encoder();
    const char* off = getenv("RGC_TC_NO_PAIR");
    g_pairs = off && std::string(off) == "1" ? 0 : std::min(resident_pairs<128>(), resident_pairs<256>());
    return true;
  }();
  (void)done;
}

bool tc_gemm_supported(const TcGemm& g) {
  if (g.m <= 0 || g.n <= 0 || g.k <= 0 || g.batch <= 0 || g.batch > (1LL << 30)) return false;
  if (g.m > (1LL << 31) || g.n > (1LL << 31) || g.k > (1LL << 31)) return false;
  return true;
}

size_t tc_gemm_scratch_bytes(const TcGemm& g) {
  Plan3 p = plan3(g);
  return p.pack_a_bytes + p.pack_b_bytes + p.part_bytes;
}

void tc_gemm(const TcGemm& g, void* scratch, int* error, cudaStream_t s) {
  Plan3 p = plan3(g);
  char* sp = (char*)scratch;
  const long long nma = g.batch_a ? g.batch : 1, nmb = g.batch_b ? g.batch : 1;
  const float* a = g.a;
  const float* b = g.b;
  long long ka = g.k, kb = g.k;  // row pitch (in K) of K-major operands
  if (p.pack_a) {
    float* d = (float*)sp;
    sp += p.pack_a_bytes;
    long long n = nma * g.m * p.kp;
    k_pack<<<(unsigned)std::max<long long>(1, std::min<long long>((n + 255) / 256, sm_count() * 8LL)), 256, 0, s>>>(d, g.a, nma, g.m, g.k, p.kp, g.batch_a, g.ta);
    a = d;
    ka = p.kp;
  }
  if (p.pack_b) {
    float* d = (float*)sp;
    sp += p.pack_b_bytes;
    long long n = nmb * g.n * p.kp;
    k_pack<<<(unsigned)std::max<long long>(1, std::min<long long>((n + 255) / 256, sm_count() * 8LL)), 256, 0, s>>>(d, g.b, nmb, g.n, g.k, p.kp, g.batch_b, !g.tb);
    b = d;
    kb = p.kp;
  }
  float* part = p.splits > 1 ? (float*)sp : nullptr;

  // Tensor maps over the operands as stored. Batch strides: packed operands are dense.
  const long long sa = p.pack_a ? g.m * p.kp : g.batch_a, sb = p.pack_b ? g.n * p.kp : g.batch_b;
  const CUtensorMapSwizzle kmaj = CU_TENSOR_MAP_SWIZZLE_128B, mnmaj = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap ma = p.a_mn ? make_map(a, g.m, g.k, nma, g.m, sa, 32, 32, mnmaj) : make_map(a, ka, g.m, nma, ka, sa, 32, BM, kmaj);
  const uint32_t b_rows = (uint32_t)(p.pair ? p.bn / 2 : p.bn);  // B rows one CTA loads
  CUtensorMap mb = p.b_mn ? make_map(b, g.n, g.k, nmb, g.n, sb, 32, 32, mnmaj) : make_map(b, kb, g.n, nmb, kb, sb, 32, b_rows, kmaj);

  Work w;
  w.M = g.m;
  w.N = g.n;
  w.mt = (int)p.mt;
  w.nt = (int)p.nt;
  w.batch = (int)g.batch;
  w.splits = p.splits;
  w.num_kb = p.num_kb;
  w.kb_per_split = p.kb_per_split;
  w.za = g.batch_a ? 1 : 0;
  w.zb = g.batch_b ? 1 : 0;
  w.C = part ? part : g.c;
  const long long units = p.mt * p.nt * g.batch * p.splits;
  if (p.pair) {
    const unsigned grid = (unsigned)(2 * std::min<long long>(units, g_pairs));
    if (p.bn == 256) launch3<256, true>(p.a_mn, p.b_mn, grid, ma, mb, w, error, s);
    else launch3<128, true>(p.a_mn, p.b_mn, grid, ma, mb, w, error, s);
  } else {
    const unsigned grid = (unsigned)std::min<long long>(units, sm_count());
    if (p.bn == 256) launch3<256, false>(p.a_mn, p.b_mn, grid, ma, mb, w, error, s);
    else if (p.bn == 128) launch3<128, false>(p.a_mn, p.b_mn, grid, ma, mb, w, error, s);
    else launch3<64, false>(p.a_mn, p.b_mn, grid, ma, mb, w, error, s);
  }
  if (part) {
    const long long count = g.batch * g.m * g.n;
    k_sum_splits<<<(unsigned)std::max<long long>(1, std::min<long long>((count + 255) / 256, sm_count() * 8LL)), 256, 0, s>>>(g.c, part, count, p.splits);
  }
}

int tc_gemm_launches(const TcGemm& g) {
  Plan3 p = plan3(g);
  return 1 + (p.pack_a ? 1 : 0) + (p.pack_b ? 1 : 0) + (p.splits > 1 ? 1 : 0);
}

}  // namespace rgc
