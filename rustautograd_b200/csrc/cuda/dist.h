// Data-parallel communicator of the CUDA device (one process per GPU). NCCL is resolved at
// run time from the library already loaded in the process (PyTorch's) or the system one, so the
// device library neither links nor pins an NCCL version.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace rgc {

bool dist_active();
// True after dist_sync aborted the communicator: the plan's all-reduce steps then fail.
bool dist_aborted();
int dist_rank();
int dist_world();
// Sum-all-reduce of `count` elements in place on `stream`; fp32 (is_f64 false) or fp64.
void dist_all_reduce(void* buf, size_t count, bool is_f64, cudaStream_t stream);
void dist_all_reduce_into(void* dst, const void* src, size_t count, bool is_f64, cudaStream_t stream);
void dist_group_start();
void dist_group_end();

// Waits for `stream`. With an active communicator the wait is bounded: after
// RGC_COLLECTIVE_TIMEOUT_S seconds (default 300) the communicator is aborted, which ends the
// collectives still waiting for another rank, and an error describing the stall is returned.
// Without one it is a plain cudaStreamSynchronize.
cudaError_t dist_sync(cudaStream_t stream, std::string* why);

}  // namespace rgc
