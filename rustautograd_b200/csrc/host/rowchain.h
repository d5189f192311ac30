// Row chains: runs of plan steps over one row space (..., C) that the CUDA device computes in
// one kernel, a block of rows at a time in shared memory (no counterpart in rg).
//
// A softmax is four plan steps over a (B, H, T, T) tensor: the masked scores, their row maximum,
// the exponentials and their row sum, and the division; each reads or writes the whole tensor.
// As a chain the scores are read once and only the values that later steps read (the
// exponentials, the probabilities, the row sums) are written. Members are elementwise steps of
// the row shape, elementwise steps of the per-row shape (..., 1), and reductions over the last
// axis with kept dimensions. Every member computes the same operations in the same order as the
// plan's own step (sums in rg's fast_sum order), so the results are the plan's, bit for bit.
#pragma once
#include <cstddef>
#include <vector>

#include "plan.h"

namespace rg {

struct RowChain {
  size_t first = 0, last = 0;       // the plan steps [first, last] the chain replaces
  std::vector<size_t> members;      // steps the chain computes, in plan order
  std::vector<size_t> before;       // other steps of the range, run before the chain, in plan order
  // Other steps of the range run after the chain: materialised broadcasts of pinned slots, whose
  // readers in the chain read the broadcast's source instead.
  std::vector<size_t> after;
  std::vector<size_t> shape;        // the row space (..., C)
  size_t rows = 0, cols = 0;
  DType dtype = DType::F32;
  // store[m][q]: output q of members[m] is written to its slot (a later step reads that slot, or
  // it is a plan output). Other values stay inside the chain.
  std::vector<std::vector<bool>> store;
};

// The chains the CUDA device forms for `plan`: unless RGC_ROW_CHAINS=0, for plans built with its
// fusion configuration (Fuse::CUDA); none otherwise. The device passes `device_plan`: the plans it
// receives across the C ABI were built for it, and the plan blob does not carry the configuration.
bool row_chains_enabled();
std::vector<RowChain> find_row_chains(const Plan& plan, bool device_plan = false);

// Slots a plan step reads and writes.
std::vector<size_t> step_reads(const Step& s);
std::vector<size_t> step_writes(const Step& s);

// Where a member step reads each of its inputs from, in the member's input order.
struct RowInput {
  enum Kind : unsigned char {
    Value,      // a value computed earlier in the chain (full or per-row, by `space`)
    Full,       // a slot holding the member's shape: element (row, j) of a full member, row of a per-row one
    Column,     // a slot holding (..., 1) read by a full member: one value per row
    Splat,      // one value
    Periodic,   // a slot repeating every `period` elements of the row space
    Broadcast,  // a slot broadcast to the member's shape by strides
    Source,     // a materialised broadcast of a pinned slot, read through its source slot `slot`
  } kind = Full;
  size_t slot = 0;
  size_t producer = 0;              // Value: index into the chain's members
  size_t output = 0;                // Value: which output of that member
  bool full_space = true;           // Value: a full value (else a per-row one)
  size_t period = 0;                // Periodic
  std::vector<size_t> shape;        // Broadcast / Source: the slot's own shape
  // Reads through a materialised broadcast (Source, or Splat / Periodic of its source): the
  // broadcast's slot, which the kernel does not read. SIZE_MAX otherwise.
  size_t through = SIZE_MAX;
};

// The inputs of member `m` of `c` (members that are not elementwise: the reduction's one input).
std::vector<RowInput> row_inputs(const Plan& plan, const RowChain& c, size_t m);

}  // namespace rg
