// Hand-written sm_100a kernels of the rg CUDA device (built with -fmad=false, IEEE division and
// square root, so single operations round exactly as rg's CPU interpreter does).
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <string>
#include <utility>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "kernels.cuh"

namespace rgc {

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("RGC_NO_PDL");
    return !(e && std::string(e) == "1");
  }();
  return on;
}

namespace {

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// Grid-stride launches use a multiple of the SM count: a few resident blocks per SM.
unsigned grid_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  long long cap = (long long)sm_count() * 8;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

// Blocks of `kernel` resident on one SM at `threads` threads per block (its registers and shared
// memory decide it), looked up once per kernel and block size.
int resident_blocks(const void* kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_tuple(kernel, threads, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, threads, smem) != cudaSuccess || nb <= 0) {
    cudaGetLastError();
    nb = 1;
  }
  cache[key] = nb;
  return nb;
}

// Programmatic dependent launch. Every kernel in this file begins with griddepcontrol.wait, which
// returns once the grids it depends on have completed and their memory is visible, so its
// launches carry the programmatic-serialization attribute. It then allows its own dependents to
// launch (griddepcontrol.launch_dependents): once all of its blocks are running, the next
// kernel's blocks are scheduled onto the SMs its finishing blocks free, and park in their own
// wait, instead of being launched after it has ended. RGC_NO_PDL=1 launches without the attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... P, typename... A>
cudaError_t launch_with(bool pdl, void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}
template <typename... P, typename... A> cudaError_t launch(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
  return launch_with(true, kernel, grid, block, smem, s, std::forward<A>(args)...);
}

// A grid-stride launch of `kernel` over n work items, covering the GPU in exactly one wave: as
// many blocks as are resident at once (fewer when n is small). A fixed 8 blocks per SM would
// leave a partial second wave for kernels that need more than 32 registers per thread.
template <typename K> unsigned grid_k(K* kernel, long long n, int threads = 256, size_t smem = 0) {
  long long b = (n + threads - 1) / threads;
  long long cap = (long long)sm_count() * resident_blocks((const void*)kernel, threads, smem);
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

template <typename T> __device__ __forceinline__ T qnan();
template <> __device__ __forceinline__ float qnan<float>() { return __int_as_float(0x7fc00000); }
template <> __device__ __forceinline__ double qnan<double>() { return __longlong_as_double(0x7ff8000000000000LL); }

template <typename T> __device__ __forceinline__ T rg_max(T a, T b) { return a > b ? a : (b >= a ? b : qnan<T>()); }
template <typename T> __device__ __forceinline__ T rg_min(T a, T b) { return a < b ? a : (b <= a ? b : qnan<T>()); }

template <typename T> __device__ __forceinline__ T combine(Red op, T acc, T x) {
  return op == Red::Sum ? acc + x : op == Red::Max ? rg_max(acc, x) : rg_min(acc, x);
}
template <typename T> __device__ __forceinline__ T red_init(Red op) {
  return op == Red::Sum ? (T)0 : op == Red::Max ? -(T)INFINITY : (T)INFINITY;
}

__device__ __forceinline__ long long clamp_index(int ix, long long dim) {
  long long v = ix < 0 ? 0 : (long long)ix;
  return v < dim - 1 ? v : dim - 1;
}

__device__ __forceinline__ unsigned long long mix(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__device__ __forceinline__ unsigned long long read_key(const int32_t* k) {
  return ((unsigned long long)(uint32_t)k[0] << 32) | (unsigned long long)(uint32_t)k[1];
}

#define GRID_STRIDE(e, n) for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < (n); e += (long long)gridDim.x * blockDim.x)

// ---------------- memory movement ----------------

template <typename T> __global__ void k_gather(T* __restrict__ dst, const T* __restrict__ src, Dims out, long long base, long long n) {
  pdl_wait();
  GRID_STRIDE(e, n) {
    long long r = e, off = base;
    for (int d = out.rank - 1; d >= 0; --d) {
      long long c = r % out.d[d];
      r /= out.d[d];
      off += c * out.st[d];
    }
    dst[e] = src[off];
  }
}

template <typename T> __global__ void k_scatter(T* __restrict__ dst, const T* __restrict__ src, Dims in, long long base, long long n) {
  pdl_wait();
  GRID_STRIDE(e, n) {
    long long r = e, off = base;
    for (int d = in.rank - 1; d >= 0; --d) {
      long long c = r % in.d[d];
      r /= in.d[d];
      off += c * in.st[d];
    }
    dst[off] = src[e];
  }
}

__device__ __forceinline__ unsigned fdiv(unsigned n, const FDiv& f) { return (__umulhi(n, f.m) + n) >> f.s; }

// Offset of element e (row-major over the extents of `s`) under the strides of `s`.
__device__ __forceinline__ long long fd_off(const FDims& s, unsigned e) {
  long long off = 0;
  for (int d = s.rank - 1; d >= 0; --d) {
    unsigned q = fdiv(e, s.d[d]);
    off += (long long)(e - q * s.d[d].d) * s.st[d];
    e = q;
  }
  return off;
}

template <typename T> __global__ void k_gather32(T* __restrict__ dst, const T* __restrict__ src, FDims s, long long base, unsigned n) {
  pdl_wait();
#pragma unroll 4
  for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) dst[e] = src[base + fd_off(s, e)];
}

template <typename T> __global__ void k_scatter32(T* __restrict__ dst, const T* __restrict__ src, FDims s, long long base, unsigned n) {
  pdl_wait();
#pragma unroll 4
  for (unsigned e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) dst[base + fd_off(s, e)] = src[e];
}

// 16-byte vectors: the innermost extent is contiguous on both sides and every offset is a
// multiple of the vector width V, so V consecutive elements move as one load and one store.
template <typename VT, int V>
__global__ void k_gather_vec(VT* __restrict__ dst, const VT* __restrict__ src, FDims s, long long base, unsigned nv) {
  pdl_wait();
  // Unrolled: with one wave of blocks each thread copies many vectors, and the loads of several
  // iterations are issued before their stores (the pointers do not alias).
#pragma unroll 4
  for (unsigned q = blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += gridDim.x * blockDim.x)
    dst[q] = src[(base + fd_off(s, q * V)) / V];
}

template <typename VT, int V>
__global__ void k_scatter_vec(VT* __restrict__ dst, const VT* __restrict__ src, FDims s, long long base, unsigned nv) {
  pdl_wait();
#pragma unroll 4
  for (unsigned q = blockIdx.x * blockDim.x + threadIdx.x; q < nv; q += gridDim.x * blockDim.x)
    dst[(base + fd_off(s, q * V)) / V] = src[q];
}

// 32x32 tiles through shared memory; the +1 column avoids bank conflicts.
template <typename T> __global__ void k_transpose2(T* __restrict__ dst, const T* __restrict__ src, long long rows, long long cols) {
  pdl_wait();
  __shared__ T tile[32][33];
  long long b = blockIdx.z;
  const T* s = src + b * rows * cols;
  T* d = dst + b * rows * cols;
  long long c0 = (long long)blockIdx.x * 32, r0 = (long long)blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    long long r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = s[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    long long c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) d[c * rows + r] = tile[threadIdx.x][i];
  }
}

// ---------------- indexing ----------------

template <typename T>
__global__ void k_take_rows(T* __restrict__ dst, const T* __restrict__ src, const int32_t* __restrict__ idx, long long dim, long long n_idx,
                            long long block, long long n) {
  pdl_wait();
  GRID_STRIDE(e, n) {
    long long row = e / block, col = e - row * block;
    long long j = row % n_idx, o = row / n_idx;
    dst[e] = src[(o * dim + clamp_index(idx[j], dim)) * block + col];
  }
}

template <typename T>
__global__ void k_take_along(T* __restrict__ dst, const T* __restrict__ src, const int32_t* __restrict__ idx, long long n, long long v, long long k) {
  pdl_wait();
  GRID_STRIDE(j, n) { dst[j] = src[(j / k) * v + clamp_index(idx[j], v)]; }
}

// One block per destination row (o, r): the block scans the indices in chunks, compacts the
// matching positions in ascending order, and every thread adds those rows for its columns in
// that order, from zero: the same sequence of additions as plan.rs:1502-1519.
template <typename T>
__global__ void k_take_grad(T* __restrict__ dst, const T* __restrict__ ct, const int32_t* __restrict__ idx, long long dim, long long n_idx,
                            long long block) {
  pdl_wait();
  __shared__ int hits[256];
  __shared__ int warp_count[8];
  __shared__ int total;
  const long long r = blockIdx.x, o = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Each thread owns columns threadIdx.x, +256, ...; block is usually <= 4 * 256.
  constexpr int MAXC = 8;
  T acc[MAXC];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) acc[c] = (T)0;
  T* out = dst + (o * dim + r) * block;
  const T* base = ct + o * n_idx * block;
  bool wide = block > 256 * MAXC;
  if (wide) {
    for (long long c = threadIdx.x; c < block; c += 256) out[c] = (T)0;
  }
  for (long long j0 = 0; j0 < n_idx; j0 += 256) {
    long long j = j0 + threadIdx.x;
    bool match = j < n_idx && clamp_index(idx[j], dim) == r;
    unsigned ballot = __ballot_sync(0xffffffffu, match);
    if (lane == 0) warp_count[warp] = __popc(ballot);
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < 8; ++w) {
        int c = warp_count[w];
        warp_count[w] = t;
        t += c;
      }
      total = t;
    }
    __syncthreads();
    if (match) hits[warp_count[warp] + __popc(ballot & ((1u << lane) - 1u))] = (int)(j - j0);
    __syncthreads();
    int m = total;
    for (int q = 0; q < m; ++q) {
      const T* row = base + (j0 + hits[q]) * block;
      if (!wide) {
#pragma unroll
        for (int c = 0; c < MAXC; ++c) {
          long long col = threadIdx.x + 256LL * c;
          if (col < block) acc[c] = acc[c] + row[col];
        }
      } else {
        for (long long col = threadIdx.x; col < block; col += 256) out[col] = out[col] + row[col];
      }
    }
    __syncthreads();
  }
  if (!wide) {
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      long long col = threadIdx.x + 256LL * c;
      if (col < block) out[col] = acc[c];
    }
  }
}

// ---- take_grad through per-row hit lists (a stable counting sort of the positions by row) ----
// Positions are cut into chunks of TG_CHUNK; cnt[r * chunks + c] counts chunk c's positions that
// land in row r. An exclusive scan of that matrix in row-major order gives where each (row,
// chunk) run starts in the list, so placing every chunk's positions in order sorts them by row
// and keeps ascending position order within a row.
constexpr int TG_CHUNK = 1024;

__global__ void k_tg_count(int* __restrict__ cnt, const int32_t* __restrict__ idx, long long dim, long long n_idx, long long chunks) {
  pdl_wait();
  GRID_STRIDE(j, n_idx) {
    long long r = clamp_index(idx[j], dim);
    atomicAdd(&cnt[r * chunks + j / TG_CHUNK], 1);
  }
}

// Exclusive scan of m values in place, one block of 1024 threads: each thread owns a contiguous run.
__global__ void k_tg_scan(int* __restrict__ v, long long m) {
  pdl_wait();
  __shared__ int part[1024];
  const long long per = (m + 1023) / 1024;
  const long long s = threadIdx.x * per, e = s + per < m ? s + per : m;
  int sum = 0;
  for (long long i = s; i < e; ++i) sum += v[i];
  part[threadIdx.x] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    int x = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
    __syncthreads();
    part[threadIdx.x] += x;
    __syncthreads();
  }
  int run = part[threadIdx.x] - sum;
  for (long long i = s; i < e; ++i) {
    int c = v[i];
    v[i] = run;
    run += c;
  }
}

// One warp per chunk, positions in ascending order 32 at a time: lanes with the same row take
// consecutive slots after that row's running offset.
__global__ void k_tg_place(int* __restrict__ list, int* __restrict__ off, const int32_t* __restrict__ idx, long long dim, long long n_idx,
                           long long chunks) {
  pdl_wait();
  const long long c = blockIdx.x;
  const int lane = threadIdx.x;
  const long long j_end = (c + 1) * TG_CHUNK < n_idx ? (c + 1) * TG_CHUNK : n_idx;
  for (long long j0 = c * TG_CHUNK; j0 < j_end; j0 += 32) {
    const long long j = j0 + lane;
    const bool live = j < j_end;
    const int r = live ? (int)clamp_index(idx[j], dim) : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, r);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (live && lane == leader) {
      base = off[(long long)r * chunks + c];
      off[(long long)r * chunks + c] = base + __popc(peers);
    }
    base = __shfl_sync(0xffffffffu, base, leader);
    if (live) list[base + __popc(peers & ((1u << lane) - 1u))] = (int)j;
    __syncwarp();
  }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
template <int N> __device__ __forceinline__ void cp_async_n(void* smem, const void* gmem) {
  unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(s), "l"(gmem), "n"(N));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Block (row r, 32-column slice, outer o): every thread stages slices of the row's hit rows into
// shared memory, TG_STAGES stages in flight; warp 0 adds them in list order (ascending
// positions), one column per lane, starting from zero.
constexpr int TG_HITS = 32;    // hit rows per stage
constexpr int TG_STAGES = 8;   // stages in flight
constexpr int TG_COLS = 32;    // columns per block

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) k_tg_accumulate(T* __restrict__ dst, const T* __restrict__ ct, const int* __restrict__ list,
                                                     const int* __restrict__ off, long long dim, long long n_idx, long long block,
                                                     long long chunks) {
  pdl_wait();
  extern __shared__ __align__(16) unsigned char tg_smem[];
  T* buf = (T*)tg_smem;  // [TG_STAGES][TG_HITS][TG_COLS]
  const long long r = blockIdx.x, o = blockIdx.z;
  const long long col0 = (long long)blockIdx.y * TG_COLS;
  const int width = (int)(block - col0 < TG_COLS ? block - col0 : TG_COLS);
  // After placement each counter holds the start of the next (row, chunk) run, so row r ends
  // at its last chunk's counter and starts where row r - 1 ends.
  const long long lo = r > 0 ? off[r * chunks - 1] : 0;
  const long long hi = off[r * chunks + chunks - 1];
  const long long m = hi - lo;
  const T* base = ct + o * n_idx * block + col0;
  const int* hits = list + lo;
  constexpr int PER = VEC ? (int)(16 / sizeof(T)) : 1;  // elements per copy
  const int copies_per_hit = (width + PER - 1) / PER;
  const long long stages = (m + TG_HITS - 1) / TG_HITS;
  auto issue = [&](long long s) {
    if (s < stages) {
      T* b = buf + (s % TG_STAGES) * TG_HITS * TG_COLS;
      const long long h0 = s * TG_HITS;
      const int nh = (int)(m - h0 < TG_HITS ? m - h0 : TG_HITS);
      for (int q = threadIdx.x; q < nh * copies_per_hit; q += blockDim.x) {
        const int h = q / copies_per_hit, k = (q - h * copies_per_hit) * PER;
        const T* src = base + (long long)hits[h0 + h] * block + k;
        if (VEC) cp_async16(b + h * TG_COLS + k, src);
        else cp_async_n<(int)sizeof(T)>(b + h * TG_COLS + k, src);
      }
    }
    cp_async_commit();
  };
  for (int s = 0; s < TG_STAGES - 1; ++s) issue(s);
  T acc = (T)0;
  const int lane = threadIdx.x;
  for (long long s = 0; s < stages; ++s) {
    issue(s + TG_STAGES - 1);
    cp_async_wait<TG_STAGES - 1>();
    __syncthreads();
    if (threadIdx.x < 32) {
      const T* b = buf + (s % TG_STAGES) * TG_HITS * TG_COLS;
      const int nh = (int)(m - s * TG_HITS < TG_HITS ? m - s * TG_HITS : TG_HITS);
      if (lane < width)
        for (int h = 0; h < nh; ++h) acc = acc + b[h * TG_COLS + lane];
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (threadIdx.x < width) dst[(o * dim + r) * block + col0 + threadIdx.x] = acc;
}

template <typename T>
__global__ void k_take_along_grad(T* __restrict__ dst, const T* __restrict__ ct, const int32_t* __restrict__ idx, long long rows, long long v,
                                  long long k) {
  pdl_wait();
  GRID_STRIDE(e, rows * v) {
    long long row = e / v, c = e - row * v;
    T acc = (T)0;
    for (long long q = 0; q < k; ++q)
      if (clamp_index(idx[row * k + q], v) == c) acc = acc + ct[row * k + q];
    dst[e] = acc;
  }
}

// ---------------- reductions ----------------

// rg's fast_sum (plan.rs:1213-1230) for n small enough to do in one warp: lanes 0..7 each add
// every eighth element in order, then lane 0 adds the eight lanes and the tail.
template <typename T> __global__ void k_sum_exact(T* dst, const T* __restrict__ a, long long n) {
  pdl_wait();
  __shared__ T lanes[8];
  int l = threadIdx.x;
  long long full = n / 8 * 8;
  if (l < 8) {
    T acc = (T)0;
    long long c = 0;
    // Loads run ahead of the dependent additions.
    for (; c + 8 * 16 <= full; c += 8 * 16) {
      T v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) v[u] = a[c + 8 * u + l];
#pragma unroll
      for (int u = 0; u < 16; ++u) acc = acc + v[u];
    }
    for (; c < full; c += 8) acc = acc + a[c + l];
    lanes[l] = acc;
  }
  __syncthreads();
  if (l == 0) {
    T out = (T)0;
    for (int k = 0; k < 8; ++k) out = out + lanes[k];
    for (long long i = full; i < n; ++i) out = out + a[i];
    dst[0] = out;
  }
}

// Fixed-order block sums: block b sums [b*chunk, (b+1)*chunk) with a fixed tree.
template <typename T> __device__ T block_sum(T v) {
  __shared__ T sh[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  int nw = (blockDim.x + 31) >> 5;
  v = threadIdx.x < nw ? sh[threadIdx.x] : (T)0;
  if (warp == 0)
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  __syncthreads();
  return v;
}

template <typename T> __global__ void k_sum_chunks(T* __restrict__ part, const T* __restrict__ a, long long n, long long chunk) {
  pdl_wait();
  long long s = (long long)blockIdx.x * chunk, e = s + chunk < n ? s + chunk : n;
  T v = (T)0;
  for (long long i = s + threadIdx.x; i < e; i += blockDim.x) v += a[i];
  v = block_sum(v);
  if (threadIdx.x == 0) part[blockIdx.x] = v;
}

template <typename T> __global__ void k_sum_final(T* dst, const T* __restrict__ part, long long m) {
  pdl_wait();
  T v = (T)0;
  for (long long i = threadIdx.x; i < m; i += blockDim.x) v += part[i];
  v = block_sum(v);
  if (threadIdx.x == 0) dst[0] = v;
}

// Warp per row for short rows, block per row for long ones.
template <typename T> __global__ void k_reduce_rows_warp(T* __restrict__ dst, const T* __restrict__ a, Red op, long long rows, long long len) {
  pdl_wait();
  long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = warp; r < rows; r += nwarps) {
    const T* row = a + r * len;
    T acc = red_init<T>(op);
    for (long long j = lane; j < len; j += 32) acc = combine(op, acc, row[j]);
    for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_down_sync(0xffffffffu, acc, o));
    if (lane == 0) dst[r] = acc;
  }
}

// Rows of 16-byte-aligned length: each lane reads 16-byte vectors (the within-row combination
// order is the vector-lane order, then the warp tree; only Sum depends on it).
template <typename T, typename VT, int V>
__global__ void k_reduce_rows_warp_vec(T* __restrict__ dst, const T* __restrict__ a, Red op, long long rows, long long len) {
  pdl_wait();
  long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long nv = len / V;
  for (long long r = warp; r < rows; r += nwarps) {
    const VT* row = (const VT*)(a + r * len);
    T acc = red_init<T>(op);
#pragma unroll 4
    for (long long j = lane; j < nv; j += 32) {
      const VT v = row[j];
      const T* e = (const T*)&v;
#pragma unroll
      for (int q = 0; q < V; ++q) acc = combine(op, acc, e[q]);
    }
    for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_down_sync(0xffffffffu, acc, o));
    if (lane == 0) dst[r] = acc;
  }
}

// Row sums in the order of rg's fast_sum (plan.rs:1213-1230): eight running sums, element j
// going to sum j % 8, then 0 + s0 + ... + s7 and the n % 8 tail in order; bit-identical to the
// CPU interpreter. Vector form: a lane owns E consecutive sums (E = elements per 16 bytes) and
// L = 8 / E lanes share a row; scalar form: one sum per lane, eight lanes per row.
template <typename T, typename VT, int E>
__global__ void k_rows_fast_sum_vec(T* __restrict__ dst, const T* __restrict__ a, long long rows, long long len) {
  pdl_wait();
  constexpr int L = 8 / E, RPW = 32 / L;
  const int lane = threadIdx.x & 31, sub = lane / L, q = lane % L;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long full = len / 8 * 8;
  for (long long r0 = warp * RPW; r0 < rows; r0 += nwarps * RPW) {
    const long long r = r0 + sub;
    T acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = (T)0;
    const T* row = a + (r < rows ? r : 0) * len;
    if (r < rows) {
      // Batches of 8 vectors loaded before they are added, so that several 16-byte loads are in
      // flight per lane; the additions into each running sum stay in element order.
      long long c = 0;
      for (; c + 64 <= full; c += 64) {
        VT v[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) v[h] = *(const VT*)(row + c + 8 * h + q * E);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const T* x = (const T*)&v[h];
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = acc[e] + x[e];
        }
      }
      for (; c < full; c += 8) {
        const VT v = *(const VT*)(row + c + q * E);
        const T* x = (const T*)&v;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = acc[e] + x[e];
      }
    }
    T out = (T)0;
#pragma unroll
    for (int k = 0; k < L; ++k)
#pragma unroll
      for (int e = 0; e < E; ++e) out = out + __shfl_sync(0xffffffffu, acc[e], sub * L + k);
    if (q == 0 && r < rows) {
      for (long long i = full; i < len; ++i) out = out + row[i];
      dst[r] = out;
    }
  }
}

template <typename T> __global__ void k_rows_fast_sum(T* __restrict__ dst, const T* __restrict__ a, long long rows, long long len) {
  pdl_wait();
  const int lane = threadIdx.x & 31, sub = lane >> 3, chain = lane & 7;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long full = len / 8 * 8;
  for (long long r0 = warp * 4; r0 < rows; r0 += nwarps * 4) {
    const long long r = r0 + sub;
    T acc = (T)0;
    const T* row = a + (r < rows ? r : 0) * len;
    if (r < rows)
      for (long long c = chain; c < full; c += 8) acc = acc + row[c];
    T out = (T)0;
#pragma unroll
    for (int k = 0; k < 8; ++k) out = out + __shfl_sync(0xffffffffu, acc, sub * 8 + k);
    if (chain == 0 && r < rows) {
      for (long long i = full; i < len; ++i) out = out + row[i];
      dst[r] = out;
    }
  }
}

template <typename T> __global__ void k_reduce_rows_block(T* __restrict__ dst, const T* __restrict__ a, Red op, long long len) {
  pdl_wait();
  __shared__ T sh[32];
  const T* row = a + (long long)blockIdx.x * len;
  T acc = red_init<T>(op);
  for (long long j = threadIdx.x; j < len; j += blockDim.x) acc = combine(op, acc, row[j]);
  for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_down_sync(0xffffffffu, acc, o));
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    int nw = blockDim.x >> 5;
    acc = lane < nw ? sh[lane] : red_init<T>(op);
    for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_down_sync(0xffffffffu, acc, o));
    if (lane == 0) dst[blockIdx.x] = acc;
  }
}

constexpr long long REDUCE_ROWS = 64;

template <typename T>
__global__ void k_cols_partial(T* __restrict__ part, const T* __restrict__ a, Red op, long long rows, long long cols) {
  pdl_wait();
  long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  long long q = blockIdx.y;
  long long r0 = q * REDUCE_ROWS, r1 = r0 + REDUCE_ROWS < rows ? r0 + REDUCE_ROWS : rows;
  T acc = red_init<T>(op);
  for (long long r = r0; r < r1; ++r) acc = combine(op, acc, a[r * cols + c]);
  part[q * cols + c] = acc;
}

// The 64-row partials with 16-byte loads: a thread folds PER adjacent columns (PER chains, each in
// row order), a full 64-row block fully unrolled so its loads are all in flight at once.
template <typename T, typename V, int PER>
__global__ void k_cols_partial_vec(T* __restrict__ part, const T* __restrict__ a, Red op, long long rows, long long cols) {
  pdl_wait();
  const long long ncv = cols / PER;
  const long long cv = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (cv >= ncv) return;
  const long long q = blockIdx.y, r0 = q * REDUCE_ROWS;
  const long long n = rows - r0 < REDUCE_ROWS ? rows - r0 : REDUCE_ROWS;
  const V* src = (const V*)(a + r0 * cols) + cv;
  T acc[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) acc[j] = red_init<T>(op);
  if (n == REDUCE_ROWS) {
    // 16 rows' loads issued before their additions, four batches per partial.
    for (int r = 0; r < (int)REDUCE_ROWS; r += 16) {
      V v[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) v[h] = src[(r + h) * ncv];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const T* e = (const T*)&v[h];
#pragma unroll
        for (int j = 0; j < PER; ++j) acc[j] = combine(op, acc[j], e[j]);
      }
    }
  } else {
    for (long long r = 0; r < n; ++r) {
      const V v = src[r * ncv];
      const T* e = (const T*)&v;
#pragma unroll
      for (int j = 0; j < PER; ++j) acc[j] = combine(op, acc[j], e[j]);
    }
  }
  V out;
  T* o = (T*)&out;
#pragma unroll
  for (int j = 0; j < PER; ++j) o[j] = acc[j];
  ((V*)(part + q * cols))[cv] = out;
}

// The final column fold: every output column folds its `nparts` rows in row order (the 64-row
// partials, or the rows themselves), one thread per column. A block owns one 32-byte sector of
// columns and stages CF_ROWS-row chunks of them in shared memory, double-buffered: the serial
// folds read shared memory while the next chunk is in flight, and the grid has a block per
// sector instead of per 32 columns.
constexpr int CF_ROWS = 1024;
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) k_cols_fold(T* __restrict__ dst, const T* __restrict__ part, Red op, long long nparts, long long cols) {
  pdl_wait();
  constexpr int C = 32 / (int)sizeof(T);  // columns per block
  constexpr int PER = VEC ? 16 / (int)sizeof(T) : 1;
  extern __shared__ __align__(16) unsigned char cf_smem[];
  T* buf = (T*)cf_smem;  // [2][CF_ROWS][C]
  const long long col0 = (long long)blockIdx.x * C;
  const int width = (int)(cols - col0 < C ? cols - col0 : C);
  const int copies = (width + PER - 1) / PER;  // per row (VEC: width is a multiple of PER)
  const long long chunks = (nparts + CF_ROWS - 1) / CF_ROWS;
  auto issue = [&](long long ch) {
    if (ch < chunks) {
      T* b = buf + (ch & 1) * CF_ROWS * C;
      const long long q0 = ch * CF_ROWS;
      const int nq = (int)(nparts - q0 < CF_ROWS ? nparts - q0 : CF_ROWS);
      for (int x = threadIdx.x; x < nq * copies; x += blockDim.x) {
        const int h = x / copies, k = (x - h * copies) * PER;
        const T* src = part + (q0 + h) * cols + col0 + k;
        if (VEC) cp_async16(b + h * C + k, src);
        else cp_async_n<(int)sizeof(T)>(b + h * C + k, src);
      }
    }
    cp_async_commit();
  };
  issue(0);
  T acc = red_init<T>(op);
  for (long long ch = 0; ch < chunks; ++ch) {
    issue(ch + 1);
    cp_async_wait<1>();
    __syncthreads();
    if (threadIdx.x < width) {
      const T* b = buf + (ch & 1) * CF_ROWS * C + threadIdx.x;
      const int nq = (int)(nparts - ch * CF_ROWS < CF_ROWS ? nparts - ch * CF_ROWS : CF_ROWS);
      int h = 0;
      for (; h + 16 <= nq; h += 16) {
        T v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = b[(h + j) * C];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = combine(op, acc, v[j]);
      }
      for (; h < nq; ++h) acc = combine(op, acc, b[h * C]);
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (threadIdx.x < width) dst[col0 + threadIdx.x] = acc;
}

template <typename T>
__global__ void k_reduce_generic(T* __restrict__ dst, const T* __restrict__ a, Red op, Dims kept, Dims red, long long n_out, long long n_red) {
  pdl_wait();
  GRID_STRIDE(o, n_out) {
    long long r = o, base = 0;
    for (int d = kept.rank - 1; d >= 0; --d) {
      long long c = r % kept.d[d];
      r /= kept.d[d];
      base += c * kept.st[d];
    }
    T acc = red_init<T>(op);
    for (long long q = 0; q < n_red; ++q) {
      long long rr = q, off = base;
      for (int d = red.rank - 1; d >= 0; --d) {
        long long c = rr % red.d[d];
        rr /= red.d[d];
        off += c * red.st[d];
      }
      acc = combine(op, acc, a[off]);
    }
    dst[o] = acc;
  }
}

// ---------------- matrix products ----------------

template <typename T, bool EXACT> __device__ __forceinline__ T mac(T acc, T a, T b);
template <> __device__ __forceinline__ float mac<float, true>(float acc, float a, float b) { return __fadd_rn(acc, __fmul_rn(a, b)); }
template <> __device__ __forceinline__ float mac<float, false>(float acc, float a, float b) { return fmaf(a, b, acc); }
template <> __device__ __forceinline__ double mac<double, true>(double acc, double a, double b) { return __dadd_rn(acc, __dmul_rn(a, b)); }
template <> __device__ __forceinline__ double mac<double, false>(double acc, double a, double b) { return fma(a, b, acc); }

// 64x64 output tile per block, 4x4 outputs per thread, k in 32-deep (f64: 16-deep) slices through
// two shared-memory buffers: the next slice's elements are loaded into registers while the current one is
// multiplied, one barrier per slice. Each output has one accumulator and k is visited in
// ascending order, so the EXACT variant performs rg's additions in rg's order.
template <typename T, bool EXACT, int TILE>
__global__ void __launch_bounds__(256) k_gemm(T* __restrict__ C, const T* __restrict__ A, const T* __restrict__ B, long long m, long long n,
                                              long long k, bool ta, bool tb, GemmBatch bt) {
  pdl_wait();
  // TILE 64: 4x4 outputs per thread; TILE 16 (small outputs, usually long k): one per thread.
  constexpr int BM = TILE, BN = TILE, R = TILE / 16;
  constexpr int BK = TILE == 16 ? 64 : (sizeof(T) == 8 ? 16 : 32);  // two buffers within 48 KB
  constexpr int LA = BM * BK / 256, LB = BK * BN / 256;             // elements per thread per slice
  __shared__ T As[2][BK][BM + 4];
  __shared__ T Bs[2][BK][BN + 4];
  long long z = blockIdx.z, oa = 0, ob = 0;
  {
    long long r = z;
    for (int d = bt.rank - 1; d >= 0; --d) {
      long long c = r % bt.d[d];
      r /= bt.d[d];
      oa += c * bt.sa[d];
      ob += c * bt.sb[d];
    }
  }
  const T* Ab = A + oa;
  const T* Bb = B + ob;
  T* Cb = C + z * m * n;
  const long long row0 = (long long)blockIdx.y * BM, col0 = (long long)blockIdx.x * BN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  T ra[LA], rb[LB];
  // Element t of a slice: A tile (i, p) = op(A)[row0 + i][k0 + p], B tile (p, j) = op(B)[k0 + p][col0 + j],
  // enumerated so that consecutive threads read consecutive addresses.
  auto load = [&](long long k0) {
#pragma unroll
    for (int q = 0; q < LA; ++q) {
      const int t = threadIdx.x + 256 * q;
      const int i = ta ? t % BM : t / BK, p = ta ? t / BM : t % BK;
      const long long gr = row0 + i, gk = k0 + p;
      ra[q] = (gr < m && gk < k) ? (ta ? Ab[gk * m + gr] : Ab[gr * k + gk]) : (T)0;
    }
#pragma unroll
    for (int q = 0; q < LB; ++q) {
      const int t = threadIdx.x + 256 * q;
      const int j = tb ? t / BK : t % BN, p = tb ? t % BK : t / BN;
      const long long gk = k0 + p, gc = col0 + j;
      rb[q] = (gk < k && gc < n) ? (tb ? Bb[gc * k + gk] : Bb[gk * n + gc]) : (T)0;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int q = 0; q < LA; ++q) {
      const int t = threadIdx.x + 256 * q;
      const int i = ta ? t % BM : t / BK, p = ta ? t / BM : t % BK;
      As[buf][p][i] = ra[q];
    }
#pragma unroll
    for (int q = 0; q < LB; ++q) {
      const int t = threadIdx.x + 256 * q;
      const int j = tb ? t / BK : t % BN, p = tb ? t % BK : t / BN;
      Bs[buf][p][j] = rb[q];
    }
  };
  T acc[R][R];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < R; ++j) acc[i][j] = (T)0;
  load(0);
  store(0);
  __syncthreads();
  int buf = 0;
  for (long long k0 = 0; k0 < k; k0 += BK) {
    const bool more = k0 + BK < k;
    if (more) load(k0 + BK);
    const int kmax = (int)(k - k0 < BK ? k - k0 : BK);
    for (int p = 0; p < kmax; ++p) {
      T av[R], bv[R];
#pragma unroll
      for (int i = 0; i < R; ++i) av[i] = As[buf][p][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < R; ++j) bv[j] = Bs[buf][p][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = mac<T, EXACT>(acc[i][j], av[i], bv[j]);
    }
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    long long r = row0 + ty + 16 * i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      long long c = col0 + tx + 16 * j;
      if (c < n) Cb[r * n + c] = acc[i][j];
    }
  }
}

// ---------------- random numbers ----------------

constexpr unsigned long long GAMMA = 0x9E3779B97F4A7C15ULL;
constexpr unsigned long long GAMMA_SPLIT = 0xD1B54A32D192ED03ULL;

__global__ void k_key_split(int32_t* dst, const int32_t* key, long long pairs) {
  pdl_wait();
  unsigned long long kk = read_key(key);
  GRID_STRIDE(j, pairs) {
    unsigned long long bits = mix(kk + (unsigned long long)(j + 1) * GAMMA_SPLIT);
    dst[2 * j] = (int32_t)(uint32_t)(bits >> 32);
    dst[2 * j + 1] = (int32_t)(uint32_t)bits;
  }
}

template <typename T> __global__ void k_rand_uniform(T* dst, const int32_t* key, long long n) {
  pdl_wait();
  unsigned long long kk = read_key(key);
  const int mant = sizeof(T) == 4 ? 24 : 53;
  const double scale = sizeof(T) == 4 ? 5.9604644775390625e-08 : 1.1102230246251565e-16;
  GRID_STRIDE(j, n) {
    unsigned long long bits = mix(kk + (unsigned long long)(j + 1) * GAMMA) >> (64 - mant);
    dst[j] = (T)((double)bits * scale);
  }
}

template <typename T> __global__ void k_rand_normal(T* dst, const int32_t* key, long long n) {
  pdl_wait();
  unsigned long long kk = read_key(key);
  const double two53 = 1.1102230246251565e-16;
  const double TAU = 6.283185307179586;
  GRID_STRIDE(j, n) {
    double u1 = 1.0 - (double)(mix(kk + (unsigned long long)(2 * j + 1) * GAMMA) >> 11) * two53;
    double u2 = (double)(mix(kk + (unsigned long long)(2 * j + 2) * GAMMA) >> 11) * two53;
    dst[j] = (T)(sqrt(-2.0 * log(u1)) * cos(TAU * u2));
  }
}

// ---------------- conversions and selection ----------------

// Rust `as` from float to i32: truncate, saturate, NaN -> 0 (plan.rs:1624-1642).
__device__ __forceinline__ int32_t to_i32(double x) {
  if (x != x) return 0;
  if (x >= 2147483647.0) return 2147483647;
  if (x <= -2147483648.0) return (int32_t)(-2147483647 - 1);
  return (int32_t)x;
}

template <typename D, typename S> __global__ void k_cast(D* dst, const S* src, long long n) {
  pdl_wait();
  GRID_STRIDE(j, n) { dst[j] = (D)src[j]; }
}
template <typename S> __global__ void k_cast_i32(int32_t* dst, const S* src, long long n) {
  pdl_wait();
  GRID_STRIDE(j, n) { dst[j] = to_i32((double)src[j]); }
}

// First index of the maximum, scanning with `x > best` (plan.rs:1437-1451): NaN never wins,
// and a NaN at index 0 wins the whole row.
template <typename T> __global__ void k_argmax(int32_t* dst, const T* __restrict__ a, long long rows, long long v) {
  pdl_wait();
  long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long r = warp; r < rows; r += nwarps) {
    const T* row = a + r * v;
    bool valid = false;
    T bv = (T)0;
    long long bi = 0;
    for (long long j = lane; j < v; j += 32) {
      T x = row[j];
      if (x != x) continue;
      if (!valid || x > bv) {
        valid = true;
        bv = x;
        bi = j;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      bool ov = __shfl_down_sync(0xffffffffu, (int)valid, o);
      T ovv = __shfl_down_sync(0xffffffffu, bv, o);
      long long oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ov && (!valid || ovv > bv || (ovv == bv && oi < bi))) {
        valid = true;
        bv = ovv;
        bi = oi;
      }
    }
    if (lane == 0) {
      T x0 = row[0];
      dst[r] = (x0 != x0 || !valid) ? 0 : (int32_t)bi;
    }
  }
}

// Rank of each element under rg's total order (larger first, ties by index, NaN last); the
// element of rank p < k is output p (plan.rs:833-866).
template <typename T> __global__ void k_arg_top_k(int32_t* dst, const T* __restrict__ a, long long v, long long k) {
  pdl_wait();
  const T* row = a + (long long)blockIdx.x * v;
  for (long long i = threadIdx.x; i < v; i += blockDim.x) {
    T p = row[i];
    bool pn = p != p;
    long long rank = 0;
    for (long long j = 0; j < v; ++j) {
      T q = row[j];
      bool qn = q != q;
      bool before;
      if (pn || qn) before = (pn != qn) ? pn : (j < i);
      else before = q > p || (q == p && j < i);
      rank += before;
    }
    if (rank < k) dst[(long long)blockIdx.x * k + rank] = (int32_t)i;
  }
}

template <typename T> __global__ void k_cumsum(T* dst, const T* __restrict__ a, long long rows, long long v, bool reverse) {
  pdl_wait();
  GRID_STRIDE(r, rows) {
    T acc = (T)0;
    if (reverse) {
      for (long long j = v - 1; j >= 0; --j) {
        acc = acc + a[r * v + j];
        dst[r * v + j] = acc;
      }
    } else {
      for (long long j = 0; j < v; ++j) {
        acc = acc + a[r * v + j];
        dst[r * v + j] = acc;
      }
    }
  }
}

__global__ void k_cumsum_i32(int32_t* dst, const int32_t* __restrict__ a, long long rows, long long v, bool reverse) {
  pdl_wait();
  GRID_STRIDE(r, rows) {
    uint32_t acc = 0;
    if (reverse) {
      for (long long j = v - 1; j >= 0; --j) dst[r * v + j] = (int32_t)(acc += (uint32_t)a[r * v + j]);
    } else {
      for (long long j = 0; j < v; ++j) dst[r * v + j] = (int32_t)(acc += (uint32_t)a[r * v + j]);
    }
  }
}

// ---------------- run loop support ----------------

__global__ void k_record_history(double* history, const void* const* slots, const int* types, int n, const long long* step, long long* bad) {
  pdl_wait();
  long long k = *step;
  bool bad_now = false;
  for (int h = 0; h < n; ++h) {
    double v;
    if (types[h] == 0) v = (double)*(const float*)slots[h];
    else if (types[h] == 1) v = *(const double*)slots[h];
    else v = (double)*(const int32_t*)slots[h];
    history[k * n + h] = v;
    bad_now = bad_now || !isfinite(v);
  }
  if (bad_now && *bad < 0) *bad = k;
}

__global__ void k_bump(long long* c) {
  pdl_wait(); *c += 1; }

__global__ void k_load_batch(char* dst, const char* batches, size_t bytes, long long nb, const long long* counter) {
  pdl_wait();
  const char* src = batches + (size_t)(*counter % nb) * bytes;
  GRID_STRIDE(i, (long long)bytes) { dst[i] = src[i]; }
}

// The condition of a conditional graph node: the scalar predicate is nonzero and, for a while
// loop, its iteration count (bumped first inside the loop body) is below the limit.
__global__ void k_set_conditional(cudaGraphConditionalHandle h, const void* pred, int dtype, long long* count, long long limit, int bump) {
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (count && bump) *count += 1;
  const double v = dtype == 0 ? (double)*(const float*)pred : dtype == 1 ? *(const double*)pred : (double)*(const int32_t*)pred;
  const bool go = v != 0.0 && (!count || *count < limit);
  cudaGraphSetConditional(h, go ? 1u : 0u);
}

__global__ void k_write_count(int32_t* dst, const long long* count) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) *dst = (int32_t)*count;
}

__global__ void k_index_outside(const int32_t* idx, long long n, long long dim, int* flag) {
  pdl_wait();
  GRID_STRIDE(i, n) {
    if (idx[i] < 0 || idx[i] >= dim) *flag = 1;
  }
}

template <typename T> __global__ void k_nonfinite(const T* a, long long n, int* flag) {
  pdl_wait();
  GRID_STRIDE(i, n) {
    if (!isfinite(a[i])) *flag = 1;
  }
}

}  // namespace

size_t esize(EType t) { return t == EType::F64 ? 8 : 4; }

void fill_zero(void* dst, size_t bytes, cudaStream_t s) { cudaMemsetAsync(dst, 0, bytes, s); }

// One segment per blockIdx.y; 16-byte vectors when both ends are 16-byte aligned.
__global__ void k_copy_segments(const Segments segs) {
  pdl_wait();
  const int g = blockIdx.y;
  const long long n = segs.count[g];
  const float* src = segs.src[g];
  float* dst = segs.dst[g];
  const long long stride = (long long)gridDim.x * blockDim.x, t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long done = 0;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    const long long n4 = n >> 2;
    for (long long i = t; i < n4; i += stride) reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    done = n4 << 2;
  }
  for (long long i = done + t; i < n; i += stride) dst[i] = src[i];
}

cudaError_t copy_segments(const Segments& segs, cudaStream_t s) {
  if (segs.n <= 0) return cudaSuccess;
  long long longest = 0;
  for (int i = 0; i < segs.n; ++i) longest = std::max(longest, segs.count[i]);
  const long long blocks = std::min<long long>((longest / 4 + 255) / 256, 256);
  return launch(k_copy_segments, dim3((unsigned)std::max<long long>(blocks, 1), (unsigned)segs.n), dim3(256), 0, s, segs);
}

#define DISPATCH(t, F, ...)                 \
  switch (t) {                              \
    case EType::F32: F<float>(__VA_ARGS__); break;  \
    case EType::F64: F<double>(__VA_ARGS__); break; \
    default: F<int32_t>(__VA_ARGS__); break;        \
  }

FDims fast_dims(const Dims& in, bool* ok) {
  // Outer to inner; a dimension folds into the next inner one when stepping it equals stepping
  // the inner one through its whole extent.
  long long d[MAXR], st[MAXR];
  int r = 0;
  *ok = true;
  for (int k = 0; k < in.rank; ++k) {
    if (in.d[k] == 1) continue;
    d[r] = in.d[k];
    st[r] = in.st[k];
    ++r;
  }
  long long md[MAXR], mst[MAXR];
  int m = 0;
  for (int k = 0; k < r; ++k) {
    if (m > 0 && mst[m - 1] == st[k] * d[k]) {
      md[m - 1] *= d[k];
      mst[m - 1] = st[k];
    } else {
      md[m] = d[k];
      mst[m] = st[k];
      ++m;
    }
  }
  FDims f;
  f.rank = m;
  for (int k = 0; k < m; ++k) {
    if (md[k] >= (1ll << 31)) *ok = false;
    f.d[k] = make_fdiv(*ok ? (unsigned long long)md[k] : 1ull);
    f.st[k] = mst[k];
  }
  return f;
}

namespace {

// Vector width (elements per 16 bytes) usable for a strided copy: the merged innermost extent
// is contiguous and every stride, the base offset and the count are multiples of it.
template <typename T> int vec_width(const FDims& f, long long base, long long n) {
  constexpr int V = (int)(16 / sizeof(T));
  if (f.rank == 0 || n % V || base % V) return 1;
  if (f.st[f.rank - 1] != 1 || f.d[f.rank - 1].d % V) return 1;
  for (int k = 0; k + 1 < f.rank; ++k)
    if (f.st[k] % V) return 1;
  return V;
}

template <typename T> struct Vec16;
template <> struct Vec16<float> { using type = float4; };
template <> struct Vec16<double> { using type = double2; };
template <> struct Vec16<int32_t> { using type = int4; };

template <typename T> void gather_t(void* dst, const void* src, const Dims& out, long long base, long long n, cudaStream_t s) {
  bool ok = false;
  FDims f = fast_dims(out, &ok);
  if (!ok || n >= (1ll << 31)) {
    launch(k_gather<T>, grid_k(k_gather<T>, n), 256, 0, s, (T*)dst, (const T*)src, out, base, n);
    return;
  }
  constexpr int V = (int)(16 / sizeof(T));
  using VT = typename Vec16<T>::type;
  if (vec_width<T>(f, base, n) == V)
    launch(k_gather_vec<VT, V>, grid_k(k_gather_vec<VT, V>, n / V), 256, 0, s, (VT*)dst, (const VT*)src, f, base, (unsigned)(n / V));
  else
    launch(k_gather32<T>, grid_k(k_gather32<T>, n), 256, 0, s, (T*)dst, (const T*)src, f, base, (unsigned)n);
}

template <typename T> void scatter_t(void* dst, const void* src, const Dims& in, long long base, long long n, cudaStream_t s) {
  bool ok = false;
  FDims f = fast_dims(in, &ok);
  if (!ok || n >= (1ll << 31)) {
    launch(k_scatter<T>, grid_k(k_scatter<T>, n), 256, 0, s, (T*)dst, (const T*)src, in, base, n);
    return;
  }
  constexpr int V = (int)(16 / sizeof(T));
  using VT = typename Vec16<T>::type;
  if (vec_width<T>(f, base, n) == V)
    launch(k_scatter_vec<VT, V>, grid_k(k_scatter_vec<VT, V>, n / V), 256, 0, s, (VT*)dst, (const VT*)src, f, base, (unsigned)(n / V));
  else
    launch(k_scatter32<T>, grid_k(k_scatter32<T>, n), 256, 0, s, (T*)dst, (const T*)src, f, base, (unsigned)n);
}

}  // namespace

void strided_gather(void* dst, const void* src, EType t, const Dims& out, long long base, long long n, cudaStream_t s) {
  if (n <= 0) return;
  DISPATCH(t, gather_t, dst, src, out, base, n, s);
}

void strided_scatter(void* dst, const void* src, EType t, const Dims& in, long long base, long long n, cudaStream_t s) {
  if (n <= 0) return;
  DISPATCH(t, scatter_t, dst, src, in, base, n, s);
}

template <typename T> static void transpose_t(void* dst, const void* src, long long batch, long long rows, long long cols, cudaStream_t s) {
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
  launch(k_transpose2<T>, grid, dim3(32, 8), 0, s, (T*)dst, (const T*)src, rows, cols);
}
void transpose_last2(void* dst, const void* src, EType t, long long batch, long long rows, long long cols, cudaStream_t s) {
  if (batch * rows * cols <= 0) return;
  DISPATCH(t, transpose_t, dst, src, batch, rows, cols, s);
}

template <typename T>
static void take_rows_t(void* dst, const void* src, const int32_t* idx, long long outer, long long dim, long long n_idx, long long block, cudaStream_t s) {
  long long n = outer * n_idx * block;
  launch(k_take_rows<T>, grid_k(k_take_rows<T>, n), 256, 0, s, (T*)dst, (const T*)src, idx, dim, n_idx, block, n);
}
void take_rows(void* dst, const void* src, const int32_t* idx, EType t, long long outer, long long dim, long long n_idx, long long block,
               cudaStream_t s) {
  if (outer * n_idx * block <= 0) return;
  DISPATCH(t, take_rows_t, dst, src, idx, outer, dim, n_idx, block, s);
}

template <typename T> static void take_along_t(void* dst, const void* src, const int32_t* idx, long long n, long long v, long long k, cudaStream_t s) {
  launch(k_take_along<T>, grid_k(k_take_along<T>, n), 256, 0, s, (T*)dst, (const T*)src, idx, n, v, k);
}
void take_along(void* dst, const void* src, const int32_t* idx, EType t, long long n, long long v, long long k, cudaStream_t s) {
  if (n <= 0) return;
  DISPATCH(t, take_along_t, dst, src, idx, n, v, k, s);
}

size_t take_grad_scratch_bytes(long long dim, long long n_idx) {
  long long chunks = (n_idx + TG_CHUNK - 1) / TG_CHUNK;
  auto a256 = [](long long b) { return (size_t)((b + 255) / 256 * 256); };
  return a256(dim * chunks * 4) + a256(n_idx * 4);
}

template <typename T, bool VEC> static void tg_accumulate(void* dst, const void* ct, const int* list, const int* off, long long outer, long long dim,
                                                           long long n_idx, long long block, long long chunks, cudaStream_t s) {
  constexpr int smem = TG_STAGES * TG_HITS * TG_COLS * (int)sizeof(T);
  static bool attr = [] {
    cudaFuncSetAttribute(k_tg_accumulate<T, VEC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    return true;
  }();
  (void)attr;
  dim3 grid((unsigned)dim, (unsigned)((block + TG_COLS - 1) / TG_COLS), (unsigned)outer);
  launch(k_tg_accumulate<T, VEC>, grid, 256, smem, s, (T*)dst, (const T*)ct, list, off, dim, n_idx, block, chunks);
}

void take_grad(void* dst, const void* ct, const int32_t* idx, EType t, long long outer, long long dim, long long n_idx, long long block,
               void* scratch, cudaStream_t s) {
  if (outer * dim * block <= 0) return;
  const long long chunks = (n_idx + TG_CHUNK - 1) / TG_CHUNK;
  const bool listed = scratch && n_idx > 0 && n_idx < (1ll << 31) && dim * chunks <= (1ll << 22) && dim < (1ll << 31) &&
                      outer <= 65535 && (block + TG_COLS - 1) / TG_COLS <= 65535;
  if (!listed) {
    dim3 grid((unsigned)dim, (unsigned)outer);
    if (t == EType::F64) launch(k_take_grad<double>, grid, 256, 0, s, (double*)dst, (const double*)ct, idx, dim, n_idx, block);
    else launch(k_take_grad<float>, grid, 256, 0, s, (float*)dst, (const float*)ct, idx, dim, n_idx, block);
    return;
  }
  int* cnt = (int*)scratch;
  int* list = (int*)((char*)scratch + (dim * chunks * 4 + 255) / 256 * 256);
  cudaMemsetAsync(cnt, 0, (size_t)(dim * chunks) * 4, s);
  launch(k_tg_count, grid_k(k_tg_count, n_idx), 256, 0, s, cnt, idx, dim, n_idx, chunks);
  launch(k_tg_scan, 1, 1024, 0, s, cnt, dim * chunks);
  launch(k_tg_place, (unsigned)chunks, 32, 0, s, list, cnt, idx, dim, n_idx, chunks);
  const bool vec = (block * (long long)esize(t)) % 16 == 0;
  if (t == EType::F64) {
    if (vec) tg_accumulate<double, true>(dst, ct, list, cnt, outer, dim, n_idx, block, chunks, s);
    else tg_accumulate<double, false>(dst, ct, list, cnt, outer, dim, n_idx, block, chunks, s);
  } else {
    if (vec) tg_accumulate<float, true>(dst, ct, list, cnt, outer, dim, n_idx, block, chunks, s);
    else tg_accumulate<float, false>(dst, ct, list, cnt, outer, dim, n_idx, block, chunks, s);
  }
}

void take_along_grad(void* dst, const void* ct, const int32_t* idx, EType t, long long rows, long long v, long long k, cudaStream_t s) {
  if (rows * v <= 0) return;
  if (t == EType::F64) launch(k_take_along_grad<double>, grid_k(k_take_along_grad<double>, rows * v), 256, 0, s, (double*)dst, (const double*)ct, idx, rows, v, k);
  else launch(k_take_along_grad<float>, grid_k(k_take_along_grad<float>, rows * v), 256, 0, s, (float*)dst, (const float*)ct, idx, rows, v, k);
}

constexpr long long EXACT_SUM_MAX = 32768;
constexpr long long SUM_CHUNK = 8192;

size_t full_sum_scratch_bytes(long long n, EType t) {
  if (n <= EXACT_SUM_MAX) return 0;
  return (size_t)((n + SUM_CHUNK - 1) / SUM_CHUNK) * esize(t);
}

cudaError_t reduce_full_sum(void* dst, const void* src, EType t, long long n, void* scratch, cudaStream_t s) {
  if (n <= EXACT_SUM_MAX) {
    if (t == EType::F64) return launch(k_sum_exact<double>, 1, 32, 0, s, (double*)dst, (const double*)src, n);
    return launch(k_sum_exact<float>, 1, 32, 0, s, (float*)dst, (const float*)src, n);
  }
  long long parts = (n + SUM_CHUNK - 1) / SUM_CHUNK;
  cudaError_t e;
  if (t == EType::F64) {
    e = launch(k_sum_chunks<double>, (unsigned)parts, 256, 0, s, (double*)scratch, (const double*)src, n, SUM_CHUNK);
    if (e != cudaSuccess) return e;
    return launch(k_sum_final<double>, 1, 1024, 0, s, (double*)dst, (const double*)scratch, parts);
  }
  e = launch(k_sum_chunks<float>, (unsigned)parts, 256, 0, s, (float*)scratch, (const float*)src, n, SUM_CHUNK);
  if (e != cudaSuccess) return e;
  return launch(k_sum_final<float>, 1, 1024, 0, s, (float*)dst, (const float*)scratch, parts);
}

template <typename T> static void rows_t(void* dst, const void* src, Red op, long long rows, long long len, cudaStream_t s) {
  if (op == Red::Sum && len <= 65536) {
    constexpr int E = (int)(16 / sizeof(T));
    using VT = typename Vec16<T>::type;
    if (len % E == 0 && ((uintptr_t)src & 15) == 0)
      launch(k_rows_fast_sum_vec<T, VT, E>, grid_k(k_rows_fast_sum_vec<T, VT, E>, rows * (8 / E)), 256, 0, s, (T*)dst, (const T*)src, rows, len);
    else
      launch(k_rows_fast_sum<T>, grid_k(k_rows_fast_sum<T>, rows * 8), 256, 0, s, (T*)dst, (const T*)src, rows, len);
    return;
  }
  if (len > 2048) {
    launch(k_reduce_rows_block<T>, (unsigned)rows, 1024, 0, s, (T*)dst, (const T*)src, op, len);
  } else {
    long long threads = rows * 32;
    constexpr int V = (int)(16 / sizeof(T));
    using VT = typename Vec16<T>::type;
    if (len % V == 0 && ((uintptr_t)src & 15) == 0)
      launch(k_reduce_rows_warp_vec<T, VT, V>, grid_k(k_reduce_rows_warp_vec<T, VT, V>, threads), 256, 0, s, (T*)dst, (const T*)src, op, rows, len);
    else
      launch(k_reduce_rows_warp<T>, grid_k(k_reduce_rows_warp<T>, threads), 256, 0, s, (T*)dst, (const T*)src, op, rows, len);
  }
}
void reduce_rows(void* dst, const void* src, EType t, Red op, long long rows, long long len, cudaStream_t s) {
  if (rows <= 0) return;
  if (t == EType::F64) rows_t<double>(dst, src, op, rows, len, s);
  else rows_t<float>(dst, src, op, rows, len, s);
}

size_t cols_scratch_bytes(long long rows, long long cols, EType t) {
  return (size_t)((rows + REDUCE_ROWS - 1) / REDUCE_ROWS) * (size_t)cols * esize(t);
}

// Every output column sums `nparts` rows of `part` in row order, staged through shared memory.
template <typename T> static void ordered_cols(void* dst, const T* part, Red op, long long nparts, long long cols, cudaStream_t s) {
  constexpr int C = 32 / (int)sizeof(T);
  constexpr int smem = 2 * CF_ROWS * 32;
  const unsigned blocks = (unsigned)((cols + C - 1) / C);
  if ((cols * (long long)sizeof(T)) % 16 == 0 && ((uintptr_t)part & 15) == 0) {
    static bool attr = (cudaFuncSetAttribute(k_cols_fold<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), true);
    (void)attr;
    launch(k_cols_fold<T, true>, blocks, 256, smem, s, (T*)dst, part, op, nparts, cols);
  } else {
    static bool attr = (cudaFuncSetAttribute(k_cols_fold<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), true);
    (void)attr;
    launch(k_cols_fold<T, false>, blocks, 256, smem, s, (T*)dst, part, op, nparts, cols);
  }
}

// rg reduces a [rows, cols] view over its rows sequentially below its parallel threshold (2^20
// elements for sums, 2^16 for max/min) and through fixed 64-row partials above it
// (plan.rs:1549-1612); both orders are kept, so sums are bit-identical.
template <typename T>
static void cols_t(void* dst, const void* src, Red op, long long rows, long long cols, bool chunked, void* scratch, cudaStream_t s) {
  // Max and min do not depend on the order: they always take the partials when large.
  const bool partials = (chunked || op != Red::Sum) && rows * cols >= (op == Red::Sum ? (1ll << 20) : (1ll << 16));
  if (!partials) {
    ordered_cols<T>(dst, (const T*)src, op, rows, cols, s);
    return;
  }
  long long parts = (rows + REDUCE_ROWS - 1) / REDUCE_ROWS;
  constexpr int PER = 16 / (int)sizeof(T);
  if (cols % PER == 0 && ((uintptr_t)src & 15) == 0 && ((uintptr_t)scratch & 15) == 0) {
    using V = typename std::conditional<sizeof(T) == 4, float4, double2>::type;
    const long long ncv = cols / PER;
    const unsigned threads = (unsigned)std::min<long long>(256, (ncv + 31) / 32 * 32);
    dim3 grid((unsigned)((ncv + threads - 1) / threads), (unsigned)parts);
    launch(k_cols_partial_vec<T, V, PER>, grid, threads, 0, s, (T*)scratch, (const T*)src, op, rows, cols);
  } else {
    dim3 grid((unsigned)((cols + 255) / 256), (unsigned)parts);
    launch(k_cols_partial<T>, grid, 256, 0, s, (T*)scratch, (const T*)src, op, rows, cols);
  }
  ordered_cols<T>(dst, (const T*)scratch, op, parts, cols, s);
}
void reduce_cols(void* dst, const void* src, EType t, Red op, long long rows, long long cols, bool chunked, void* scratch, cudaStream_t s) {
  if (cols <= 0) return;
  if (t == EType::F64) cols_t<double>(dst, src, op, rows, cols, chunked, scratch, s);
  else cols_t<float>(dst, src, op, rows, cols, chunked, scratch, s);
}

void reduce_generic(void* dst, const void* src, EType t, Red op, const Dims& kept, const Dims& reduced, long long n_out, cudaStream_t s) {
  if (n_out <= 0) return;
  long long n_red = 1;
  for (int d = 0; d < reduced.rank; ++d) n_red *= reduced.d[d];
  if (t == EType::F64) launch(k_reduce_generic<double>, grid_k(k_reduce_generic<double>, n_out), 256, 0, s, (double*)dst, (const double*)src, op, kept, reduced, n_out, n_red);
  else launch(k_reduce_generic<float>, grid_k(k_reduce_generic<float>, n_out), 256, 0, s, (float*)dst, (const float*)src, op, kept, reduced, n_out, n_red);
}

void gemm(void* c, const void* a, const void* b, EType t, long long m, long long n, long long k, bool ta, bool tb, const GemmBatch& batch,
          long long count, bool exact, cudaStream_t s) {
  if (m * n * count <= 0) return;
  if (k == 0) {
    cudaMemsetAsync(c, 0, (size_t)(m * n * count) * esize(t), s);
    return;
  }
  // 16x16 tiles (one output per thread) when 64x64 tiles would not fill the GPU once.
  const bool small = ((n + 63) / 64) * ((m + 63) / 64) * count < sm_count();
  const long long tile = small ? 16 : 64;
  dim3 grid((unsigned)((n + tile - 1) / tile), (unsigned)((m + tile - 1) / tile), (unsigned)count);
  auto run = [&](auto kernel, auto* cc, auto* aa, auto* bb) { launch(kernel, grid, 256, 0, s, cc, aa, bb, m, n, k, ta, tb, batch); };
  if (t == EType::F64) {
    auto *cc = (double*)c, *aa = (double*)a, *bb = (double*)b;
    if (small) exact ? run(k_gemm<double, true, 16>, cc, aa, bb) : run(k_gemm<double, false, 16>, cc, aa, bb);
    else exact ? run(k_gemm<double, true, 64>, cc, aa, bb) : run(k_gemm<double, false, 64>, cc, aa, bb);
  } else {
    auto *cc = (float*)c, *aa = (float*)a, *bb = (float*)b;
    if (small) exact ? run(k_gemm<float, true, 16>, cc, aa, bb) : run(k_gemm<float, false, 16>, cc, aa, bb);
    else exact ? run(k_gemm<float, true, 64>, cc, aa, bb) : run(k_gemm<float, false, 64>, cc, aa, bb);
  }
}

void key_split(int32_t* dst, const int32_t* key, long long pairs, cudaStream_t s) {
  if (pairs <= 0) return;
  launch(k_key_split, grid_k(k_key_split, pairs), 256, 0, s, dst, key, pairs);
}

void rand_uniform(void* dst, const int32_t* key, EType t, long long n, cudaStream_t s) {
  if (n <= 0) return;
  if (t == EType::F64) launch(k_rand_uniform<double>, grid_k(k_rand_uniform<double>, n), 256, 0, s, (double*)dst, key, n);
  else launch(k_rand_uniform<float>, grid_k(k_rand_uniform<float>, n), 256, 0, s, (float*)dst, key, n);
}

void rand_normal(void* dst, const int32_t* key, EType t, long long n, cudaStream_t s) {
  if (n <= 0) return;
  if (t == EType::F64) launch(k_rand_normal<double>, grid_k(k_rand_normal<double>, n), 256, 0, s, (double*)dst, key, n);
  else launch(k_rand_normal<float>, grid_k(k_rand_normal<float>, n), 256, 0, s, (float*)dst, key, n);
}

void cast(void* dst, EType dt, const void* src, EType st, long long n, cudaStream_t s) {
  if (n <= 0) return;
  unsigned g = grid_for(n);
  if (dt == EType::F32 && st == EType::F64) launch(k_cast<float, double>, g, 256, 0, s, (float*)dst, (const double*)src, n);
  else if (dt == EType::F64 && st == EType::F32) launch(k_cast<double, float>, g, 256, 0, s, (double*)dst, (const float*)src, n);
  else if (dt == EType::F32 && st == EType::I32) launch(k_cast<float, int32_t>, g, 256, 0, s, (float*)dst, (const int32_t*)src, n);
  else if (dt == EType::F64 && st == EType::I32) launch(k_cast<double, int32_t>, g, 256, 0, s, (double*)dst, (const int32_t*)src, n);
  else if (dt == EType::I32 && st == EType::F32) launch(k_cast_i32<float>, g, 256, 0, s, (int32_t*)dst, (const float*)src, n);
  else if (dt == EType::I32 && st == EType::F64) launch(k_cast_i32<double>, g, 256, 0, s, (int32_t*)dst, (const double*)src, n);
}

void argmax(int32_t* dst, const void* src, EType t, long long rows, long long v, cudaStream_t s) {
  if (rows <= 0) return;
  if (t == EType::F64) launch(k_argmax<double>, grid_k(k_argmax<double>, rows * 32), 256, 0, s, dst, (const double*)src, rows, v);
  else launch(k_argmax<float>, grid_k(k_argmax<float>, rows * 32), 256, 0, s, dst, (const float*)src, rows, v);
}

void arg_top_k(int32_t* dst, const void* src, EType t, long long rows, long long v, long long k, cudaStream_t s) {
  if (rows <= 0) return;
  if (t == EType::F64) launch(k_arg_top_k<double>, (unsigned)rows, 256, 0, s, dst, (const double*)src, v, k);
  else launch(k_arg_top_k<float>, (unsigned)rows, 256, 0, s, dst, (const float*)src, v, k);
}

void cumsum(void* dst, const void* src, EType t, long long rows, long long v, bool reverse, cudaStream_t s) {
  if (rows <= 0 || v <= 0) return;
  unsigned g = grid_for(rows, 128);
  if (t == EType::F64) launch(k_cumsum<double>, g, 128, 0, s, (double*)dst, (const double*)src, rows, v, reverse);
  else if (t == EType::F32) launch(k_cumsum<float>, g, 128, 0, s, (float*)dst, (const float*)src, rows, v, reverse);
  else launch(k_cumsum_i32, g, 128, 0, s, (int32_t*)dst, (const int32_t*)src, rows, v, reverse);
}

void record_history(double* history, const void* const* slots, const int* types, int n, const long long* step, long long* bad_step,
                    cudaStream_t s) {
  launch(k_record_history, 1, 1, 0, s, history, slots, types, n, step, bad_step);
}

void bump_counter(long long* counter, cudaStream_t s) { launch(k_bump, 1, 1, 0, s, counter); }

void load_batch(void* dst, const void* batches, size_t bytes, long long n_batches, const long long* counter, cudaStream_t s) {
  launch(k_load_batch, grid_k(k_load_batch, (long long)bytes), 256, 0, s, (char*)dst, (const char*)batches, bytes, n_batches, counter);
}

void set_conditional(cudaGraphConditionalHandle h, const void* pred, EType t, long long* count, long long limit, bool bump, cudaStream_t s) {
  // The kernel that sets a conditional graph node's condition keeps a plain launch.
  launch_with(false, k_set_conditional, 1, 32, 0, s, h, pred, (int)t, count, limit, bump ? 1 : 0);
}

void write_count(int32_t* dst, const long long* count, cudaStream_t s) { launch(k_write_count, 1, 32, 0, s, dst, count); }

void index_outside(const int32_t* idx, long long n, long long dim, int* flag, cudaStream_t s) {
  if (n <= 0) return;
  launch(k_index_outside, grid_k(k_index_outside, n), 256, 0, s, idx, n, dim, flag);
}

void any_nonfinite(const void* src, EType t, long long n, int* flag, cudaStream_t s) {
  if (n <= 0) return;
  if (t == EType::F64) launch(k_nonfinite<double>, grid_k(k_nonfinite<double>, n), 256, 0, s, (const double*)src, n, flag);
  else if (t == EType::F32) launch(k_nonfinite<float>, grid_k(k_nonfinite<float>, n), 256, 0, s, (const float*)src, n, flag);
}

}  // namespace rgc
