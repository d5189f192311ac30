// A row chain (rowchain.h) as one generated kernel. Each block of threads takes a block of rows
// and runs the chain's stages over it in order, with a barrier between stages: a stage is a run
// of full elementwise members (one pass over the block's elements, values in registers), a run of
// per-row members (one pass over its rows), or one reduction along the rows. Full-size values a
// later stage reads are kept in shared memory (one row pitch apart); per-row values always are.
// Only the values the chain stores are written to their slots.
//
// Per element every member evaluates the same expressions as the plan's own kernels (jit.cpp).
// Sums follow rg's fast_sum (plan.rs:1213-1230): eight running sums over the row, element j into
// sum j % 8 in order, then 0 + s0 + ... + s7 and the row's last len % 8 elements in order. Maxima
// and minima equal rg's sequential fold (nan_max / nan_min from -inf / +inf): the extreme value,
// canonical NaN if any element is NaN, and among equal extremes (-0 and +0) the last one's bits;
// eight lanes fold their classes in order and the lane results are combined by value and index.
#pragma once
#include <string>
#include <vector>

#include "jit.h"
#include "rowchain.h"

namespace rgc {

struct RowKernel {
  std::string name, source;
  std::vector<size_t> in_slots;   // ElemArgs::in[k]
  std::vector<FDiv> in_div;       // ElemArgs::row[k]: the period of a periodic input
  std::vector<size_t> out_slots;  // ElemArgs::out[q]
  std::vector<FDims> bcs;         // broadcast descriptors, ElemArgs::bc[...] from the kernel's base
  long long rows = 0;
  int rows_per_block = 0;
  size_t smem = 0;                // dynamic shared memory per block, bytes
};

constexpr int ROW_THREADS = 256;

// Builds the kernel for chain `c` of `plan`; false (with `why`) when it cannot (an index or a
// broadcast that does not fit the 32-bit path, or a block that does not fit shared memory).
bool make_row_kernel(const rg::Plan& plan, const rg::RowChain& c, RowKernel* k, std::string* why);

}  // namespace rgc
