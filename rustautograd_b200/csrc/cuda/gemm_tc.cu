// fp32-accurate GEMM on sm_100a tensor cores: 3xTF32 with tcgen05.mma, TMEM accumulators and a
// TMA-fed, mbarrier-synchronised shared-memory pipeline (no cluster multicast).
//
// Each fp32 operand x is split once, before the product, into hi = tf32(x) (rounded, low 13 bits
// zero) and lo = x - hi; C = A_hi B_hi + A_hi B_lo + A_lo B_hi, accumulated in fp32 in TMEM. The
// dropped A_lo B_lo term and the truncation of lo to TF32 leave a relative error near 1e-6,
// well inside the 1e-4 parity bound.
//
// Tile: 128 (M) x BN (N) x 32 (K) per stage, 3 stages. The split pre-pass writes both operands
// K-major whatever their layout in memory (ta/tb), so TMA always fills 128-byte-swizzled K-major
// tiles and the MMA always runs in its K-major x K-major form. Warp 0 lane 0 issues TMA, warp 1 lane 0 issues MMAs, all four warps
// drain the accumulator (each warp owns 32 TMEM lanes = 32 rows). Every wait is bounded by a
// wall-clock limit; on expiry the kernel records an error code and exits cleanly.
#include <cuda.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "gemm_tc.cuh"

namespace rgc {

namespace {

constexpr int BM = 128, BK = 32, STAGES = 3;
constexpr uint32_t A_TILE = BM * BK * 4;  // 16 KB
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

// Waits for `phase` of `bar`; gives up after WAIT_LIMIT_NS or when another role aborted.
__device__ bool mbar_wait(uint64_t* bar, uint32_t phase, volatile int* abort, int* err, int code) {
  unsigned long long t0 = now_ns();
  for (;;) {
    if (mbar_try(bar, phase)) return true;
    if (*abort) return false;
    if (now_ns() - t0 > WAIT_LIMIT_NS) {
      *abort = 1;
      atomicExch(err, code);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(saddr(dst)),
      "l"(map), "r"(saddr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Shared-memory matrix descriptors (tcgen05 "matrix descriptor", version 1, 128-byte swizzle).
// K-major: rows of 32 fp32 (128 B), 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;             // descriptor version
  d |= (uint64_t)2 << 61;             // 128-byte swizzle
  return d;
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  const uint32_t no_mask = 0;  // disable-output-lane mask: every lane written
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(no_mask)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar)) : "memory");
}

__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,"
      "%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]),
        "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
        "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
        "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN>
__global__ void __launch_bounds__(128, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl, const __grid_constant__ CUtensorMap mBh,
              const __grid_constant__ CUtensorMap mBl, float* __restrict__ C, long long M, long long N, int num_kb, int za, int zb, int* err) {
  constexpr uint32_t B_TILE = BN * BK * 4;
  constexpr uint32_t STAGE = 2 * A_TILE + 2 * B_TILE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(accum + 1);
  volatile int* abort = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int z = blockIdx.z;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)), "r"((uint32_t)BN) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  // Instruction descriptor: M = 128, N = BN, TF32 x TF32 -> F32, both operands K-major.
  const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

  if (threadIdx.x == 0) {
    // Producer: one stage = A hi, A lo, B hi, B lo for one 32-wide slice of K.
    int issued = 0;
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % STAGES;
      if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, abort, err, 1)) break;
      mbar_expect_tx(&full[s], STAGE);
      uint8_t* st = smem + s * STAGE;
      const int k0 = kb * BK;
      tma_load(st, &mAh, &full[s], k0, m0, z * za);
      tma_load(st + A_TILE, &mAl, &full[s], k0, m0, z * za);
      uint8_t* sb = st + 2 * A_TILE;
      tma_load(sb, &mBh, &full[s], k0, n0, z * zb);
      tma_load(sb + B_TILE, &mBl, &full[s], k0, n0, z * zb);
      issued = kb + 1;
    }
    if (*abort) {
      // Let the copies already in flight land before the block's shared memory goes away.
      for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb) {
        unsigned long long t0 = now_ns();
        while (!mbar_try(&full[kb % STAGES], (kb / STAGES) & 1) && now_ns() - t0 < WAIT_LIMIT_NS) {
        }
      }
    }
  } else if (threadIdx.x == 32) {
    // MMA issuer: three TF32 products per 8-deep K step into the TMEM accumulator.
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&full[s], (kb / STAGES) & 1, abort, err, 2)) break;
      fence_after();
      const uint32_t sa = saddr(smem + s * STAGE);
      const uint32_t sb = sa + 2 * A_TILE;
#pragma unroll
      for (int kk = 0; kk < BK / 8; ++kk) {
        // K advances 8 fp32 = 32 bytes within the 128-byte swizzle row.
        const uint64_t ah = desc_k(sa + kk * 32), al = desc_k(sa + A_TILE + kk * 32);
        const uint64_t bh = desc_k(sb + kk * 32), bl = desc_k(sb + B_TILE + kk * 32);
        mma_tf32(tmem, ah, bh, idesc, (kb | kk) != 0);
        mma_tf32(tmem, ah, bl, idesc, 1);
        mma_tf32(tmem, al, bh, idesc, 1);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(accum);  // also after an abort: the epilogue waits for the products in flight
  }
  __syncwarp();

  // Epilogue: warp w drains TMEM lanes [32w, 32w + 32) = rows m0 + 32w + lane.
  bool ok = mbar_wait(accum, 0, abort, err, 3);
  fence_after();
  const long long row = m0 + warp * 32 + lane;
  if (ok && !*abort) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
      if (row < M) {
        float* out = C + (long long)z * M * N + row * N + n0 + c;
        const long long lim = N - (n0 + c);
        if (lim >= 32 && (((uintptr_t)out & 15) == 0)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) *(float4*)(out + j) = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < lim) out[j] = __uint_as_float(v[j]);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

__device__ __forceinline__ void split1(float v, float* hi, float* lo) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
  *hi = __uint_as_float(h);
  *lo = v - *hi;
}

// Operand preparation, K-major: out[z][r][k] for r < R, k < Kp (zero for k >= K), with
// hi = round-to-nearest TF32 of the value (low 13 bits zero) and lo = value - hi.
// Source element (z, r, k) is src[z * sz + r * K + k].
__global__ void k_split_rows(float* __restrict__ hi, float* __restrict__ lo, const float* __restrict__ src, long long nmat, long long R,
                             long long K, long long Kp, long long sz) {
  const long long n = nmat * R * Kp;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    long long k = e % Kp, rz = e / Kp, r = rz % R, z = rz / R;
    float v = k < K ? src[z * sz + r * K + k] : 0.f;
    split1(v, hi + e, lo + e);
  }
}

// The same from a source stored transposed: element (z, r, k) is src[z * sz + k * R + r].
// 32 x 32 tiles through shared memory keep both the reads and the writes coalesced.
__global__ void k_split_cols(float* __restrict__ hi, float* __restrict__ lo, const float* __restrict__ src, long long R, long long K, long long Kp,
                             long long sz) {
  __shared__ float tile[32][33];
  const long long z = blockIdx.z;
  const long long r0 = (long long)blockIdx.x * 32, k0 = (long long)blockIdx.y * 32;
  const float* s = src + z * sz;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    long long k = k0 + i, r = r0 + threadIdx.x;
    tile[i][threadIdx.x] = (k < K && r < R) ? s[k * R + r] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    long long r = r0 + i, k = k0 + threadIdx.x;
    if (r < R && k < Kp) {
      long long o = (z * R + r) * Kp + k;
      split1(tile[threadIdx.x][i], hi + o, lo + o);
    }
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
                     uint32_t box_inner, uint32_t box_outer) {
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(row_stride * 4), (cuuint64_t)(batch_stride * 4)};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed (CUresult " + std::to_string((int)r) + ")");
  return m;
}

int pick_bn(long long n) { return n >= 96 ? 128 : n > 32 ? 64 : 32; }

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

void tc_gemm_init() {
  static bool done = [] {
    for (int bn : {32, 64, 128}) {
      size_t smem = 1024 + STAGES * (2 * A_TILE + 2 * (size_t)bn * BK * 4) + 256;
      cudaError_t e = bn == 128 ? cudaFuncSetAttribute(k_tc_gemm<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                      : bn == 64 ? cudaFuncSetAttribute(k_tc_gemm<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
                                 : cudaFuncSetAttribute(k_tc_gemm<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) throw std::runtime_error(std::string("tensor-core GEMM setup failed: ") + cudaGetErrorString(e));
    }
    encoder();
    return true;
  }();
  (void)done;
}

bool tc_gemm_supported(const TcGemm& g) {
  if (g.m <= 0 || g.n <= 0 || g.k <= 0 || g.batch <= 0 || g.batch > 65535) return false;
  if (g.m > (1LL << 31) || g.n > (1LL << 31) || g.k > (1LL << 31)) return false;
  return true;
}

namespace {
long long kpad(long long k) { return (k + 3) / 4 * 4; }  // a K-major row of Kp floats is 16-byte aligned
}  // namespace

size_t tc_gemm_scratch_bytes(const TcGemm& g) {
  long long nma = g.batch_a ? g.batch : 1, nmb = g.batch_b ? g.batch : 1, kp = kpad(g.k);
  return 2 * (align256((size_t)(nma * g.m * kp) * 4) + align256((size_t)(nmb * g.n * kp) * 4));
}

void tc_gemm(const TcGemm& g, void* scratch, int* error, cudaStream_t s) {
  // Both operands are first written K-major (hi and lo halves, K padded to a multiple of 4 with
  // zeros): the product then always runs in the K-major x K-major MMA form.
  const int za = g.batch_a ? 1 : 0, zb = g.batch_b ? 1 : 0;
  const long long nma = za ? g.batch : 1, nmb = zb ? g.batch : 1, kp = kpad(g.k);
  char* p = (char*)scratch;
  float* ah = (float*)p;
  p += align256((size_t)(nma * g.m * kp) * 4);
  float* al = (float*)p;
  p += align256((size_t)(nma * g.m * kp) * 4);
  float* bh = (float*)p;
  p += align256((size_t)(nmb * g.n * kp) * 4);
  float* bl = (float*)p;
  static int sms = [] {
    int d = 0, v = 148;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    return v;
  }();
  // rows x K matrices, `trans`: stored [K, rows] instead of [rows, K].
  auto prepare = [&](float* hi, float* lo, const float* x, long long nmat, long long rows, long long sz, bool trans) {
    if (trans) {
      dim3 grid((unsigned)((rows + 31) / 32), (unsigned)((kp + 31) / 32), (unsigned)nmat);
      k_split_cols<<<grid, dim3(32, 8), 0, s>>>(hi, lo, x, rows, g.k, kp, sz);
    } else {
      long long n = nmat * rows * kp;
      long long blocks = std::min<long long>((n + 255) / 256, (long long)sms * 8);
      k_split_rows<<<(unsigned)std::max<long long>(blocks, 1), 256, 0, s>>>(hi, lo, x, nmat, rows, g.k, kp, sz);
    }
  };
  prepare(ah, al, g.a, nma, g.m, g.batch_a, g.ta);
  prepare(bh, bl, g.b, nmb, g.n, g.batch_b, !g.tb);

  const int bn = pick_bn(g.n);
  CUtensorMap mah = make_map(ah, kp, g.m, nma, kp, g.m * kp, 32, BM);
  CUtensorMap mal = make_map(al, kp, g.m, nma, kp, g.m * kp, 32, BM);
  CUtensorMap mbh = make_map(bh, kp, g.n, nmb, kp, g.n * kp, 32, (uint32_t)bn);
  CUtensorMap mbl = make_map(bl, kp, g.n, nmb, kp, g.n * kp, 32, (uint32_t)bn);
  const int num_kb = (int)((kp + BK - 1) / BK);
  dim3 grid((unsigned)((g.n + bn - 1) / bn), (unsigned)((g.m + BM - 1) / BM), (unsigned)g.batch);
  const size_t stage = 2 * A_TILE + 2 * (size_t)bn * BK * 4;
  const size_t smem = 1024 + STAGES * stage + 256;
  auto launch = [&](auto kernel) { kernel<<<grid, 128, smem, s>>>(mah, mal, mbh, mbl, g.c, g.m, g.n, num_kb, za, zb, error); };
  if (bn == 128) launch(k_tc_gemm<128>);
  else if (bn == 64) launch(k_tc_gemm<64>);
  else launch(k_tc_gemm<32>);
}

}  // namespace rgc
