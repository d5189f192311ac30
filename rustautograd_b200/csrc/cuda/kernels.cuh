// Host-side launchers for the hand-written sm_100a kernels of the rg CUDA device.
// Every kernel is deterministic: the same inputs give the same bits on every run, which the
// device-resident run loop relies on to replay a chunk of steps exactly.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace rgc {

constexpr int MAXR = 8;  // largest tensor rank the index kernels handle

struct Dims {
  int rank = 0;
  long long d[MAXR] = {};   // extents
  long long st[MAXR] = {};  // strides (elements) paired with the extents
};

// Division by a runtime-invariant divisor d in [1, 2^31] for dividends below 2^31, as a multiply
// and shift (the round-up method of Granlund and Montgomery, "Division by invariant integers
// using multiplication", PLDI 1994): with s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> s. Index kernels use it instead of 64-bit division.
struct FDiv {
  unsigned d = 1, m = 1, s = 0;
};
inline FDiv make_fdiv(unsigned long long d) {
  FDiv f;
  f.d = (unsigned)d;
  unsigned s = 0;
  while ((1ull << s) < d) ++s;
  f.s = s;
  f.m = (unsigned)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  return f;
}

// Dims with extents as fast divisors, adjacent dimensions merged where the memory order allows
// and extents of 1 dropped (rank 0 = a single element). Valid when every extent and the element
// count are below 2^31.
struct FDims {
  int rank = 0;
  FDiv d[MAXR];
  long long st[MAXR] = {};
};
// Merges and converts; `ok` is false when some extent is 2^31 or more.
FDims fast_dims(const Dims& in, bool* ok);

enum class EType : int { F32 = 0, F64 = 1, I32 = 2 };

size_t esize(EType t);

// ---- memory movement ----
// Whether launches carry the programmatic-dependent-launch attribute (off with RGC_NO_PDL=1).
bool pdl_enabled();
void fill_zero(void* dst, size_t bytes, cudaStream_t s);
// dst[e] = src[base + sum_d coord_d(e) * src.st[d]] over the output extents `out.d`.
void strided_gather(void* dst, const void* src, EType t, const Dims& out, long long base, long long n, cudaStream_t s);
// dst[base + sum_d coord_d(e) * dst.st[d]] = src[e] over the input extents `in.d`.
void strided_scatter(void* dst, const void* src, EType t, const Dims& in, long long base, long long n, cudaStream_t s);
// Tiled transpose of the last two axes of a [batch, rows, cols] view: dst[b][c][r] = src[b][r][c].
void transpose_last2(void* dst, const void* src, EType t, long long batch, long long rows, long long cols, cudaStream_t s);

// ---- indexing (plan.rs:1365-1389, 1502-1531) ----
void take_rows(void* dst, const void* src, const int32_t* idx, EType t, long long outer, long long dim, long long n_idx,
               long long block, cudaStream_t s);
void take_along(void* dst, const void* src, const int32_t* idx, EType t, long long n, long long v, long long k, cudaStream_t s);
// Deterministic scatter-add: each destination row sums its contributions in ascending index
// order starting from zero, the order rg's sequential loop adds them. The positions are first
// sorted by row into per-row hit lists in `scratch` (take_grad_scratch_bytes bytes).
size_t take_grad_scratch_bytes(long long dim, long long n_idx);
void take_grad(void* dst, const void* ct, const int32_t* idx, EType t, long long outer, long long dim, long long n_idx,
               long long block, void* scratch, cudaStream_t s);
void take_along_grad(void* dst, const void* ct, const int32_t* idx, EType t, long long rows, long long v, long long k,
                     cudaStream_t s);

// ---- reductions (plan.rs:1549-1622) ----
enum class Red : int { Sum = 0, Max = 1, Min = 2 };
// Full sum in rg's eight-lane order (bit-exact) for small n; a fixed-order tree otherwise.
// `scratch` needs full_sum_scratch_bytes(n) bytes.
size_t full_sum_scratch_bytes(long long n, EType t);
// Returns the first launch error (the launches' own status, not cudaGetLastError).
cudaError_t reduce_full_sum(void* dst, const void* src, EType t, long long n, void* scratch, cudaStream_t s);
// Rows of length `len` reduced to one value each.
void reduce_rows(void* dst, const void* src, EType t, Red op, long long rows, long long len, cudaStream_t s);
// [rows, cols] reduced over rows in rg's order: sequentially, or, when `chunked` (rg's own
// pattern test for its parallel path) and the input reaches rg's parallel threshold, through
// fixed 64-row partials (plan.rs:1593-1612) kept in `scratch` (cols_scratch_bytes bytes).
size_t cols_scratch_bytes(long long rows, long long cols, EType t);
void reduce_cols(void* dst, const void* src, EType t, Red op, long long rows, long long cols, bool chunked, void* scratch, cudaStream_t s);
// Anything else: one output per thread, reduced coordinates walked in row-major order.
void reduce_generic(void* dst, const void* src, EType t, Red op, const Dims& kept, const Dims& reduced, long long n_out,
                    cudaStream_t s);

// ---- matrix products (tensor.rs:238-251, plan.rs:1453-1493) ----
struct GemmBatch {
  int rank = 0;
  long long d[MAXR] = {};
  long long sa[MAXR] = {}, sb[MAXR] = {};  // per-batch-dim element strides of A and B (0 = broadcast)
};
// C[b] (m x n) = op(A[b]) @ op(B[b]); `exact` keeps rg's loop arithmetic (k ascending, separate
// multiply and add roundings), so results are bit-identical to the CPU interpreter.
void gemm(void* c, const void* a, const void* b, EType t, long long m, long long n, long long k, bool ta, bool tb,
          const GemmBatch& batch, long long count, bool exact, cudaStream_t s);

// ---- random numbers (plan.rs:1403-1435, 1532-1544) ----
void key_split(int32_t* dst, const int32_t* key, long long pairs, cudaStream_t s);
void rand_uniform(void* dst, const int32_t* key, EType t, long long n, cudaStream_t s);
void rand_normal(void* dst, const int32_t* key, EType t, long long n, cudaStream_t s);

// ---- conversions and per-row selection ----
void cast(void* dst, EType dt, const void* src, EType st, long long n, cudaStream_t s);
void argmax(int32_t* dst, const void* src, EType t, long long rows, long long v, cudaStream_t s);
void arg_top_k(int32_t* dst, const void* src, EType t, long long rows, long long v, long long k, cudaStream_t s);
void cumsum(void* dst, const void* src, EType t, long long rows, long long v, bool reverse, cudaStream_t s);

// ---- run loop support ----
// history[step * n + h] = (double) slot_h[0]; sets *bad_step (if still -1) when not finite.
void record_history(double* history, const void* const* slots, const int* types, int n, const long long* step,
                    long long* bad_step, cudaStream_t s);
void bump_counter(long long* counter, cudaStream_t s);
// Loads batch (*counter % n_batches) of a data input from the device-resident batch array.
void load_batch(void* dst, const void* batches, size_t bytes, long long n_batches, const long long* counter, cudaStream_t s);
// Any non-finite value in a float buffer -> *flag = 1.
void any_nonfinite(const void* src, EType t, long long n, int* flag, cudaStream_t s);
// Control flow in CUDA graphs: sets conditional node `h` from a scalar predicate (and, with
// `count`, the iteration count below `limit`; `bump` first adds one to it); the count as int32.
void set_conditional(cudaGraphConditionalHandle h, const void* pred, EType t, long long* count, long long limit, bool bump, cudaStream_t s);
void write_count(int32_t* dst, const long long* count, cudaStream_t s);
// Any index outside [0, dim) -> *flag = 1.
void index_outside(const int32_t* idx, long long n, long long dim, int* flag, cudaStream_t s);

// Up to SEGMENTS_MAX float segments copied in one launch (the gradients of a data-parallel
// step gathered into one contiguous buffer for a single all-reduce, and scattered back).
constexpr int SEGMENTS_MAX = 64;
struct Segments {
  int n = 0;
  const float* src[SEGMENTS_MAX];
  float* dst[SEGMENTS_MAX];
  long long count[SEGMENTS_MAX];
};
cudaError_t copy_segments(const Segments& segs, cudaStream_t s);

}  // namespace rgc
