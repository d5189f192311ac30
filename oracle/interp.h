// TEST INFRASTRUCTURE — the parity oracle and the timed CPU baseline, never a product path.
//
// A CPU restatement of rg's plan interpreter (src/plan.rs:657-1642 and the portable kernels of
// src/tensor.rs:200-251): the same block/task chunking, thresholds, per-element arithmetic order,
// naive GEMM loop order and glibc libm calls that rg uses on Linux. Only tests/, the smoke check
// and bench.py's CPU-baseline leg load it.
#pragma once
#include <functional>

#include "../rustautograd_b200/csrc/host/exec.h"

namespace rg::oracle {

// The cross-rank sum behind the `all_reduce` op (data parallelism). Without a hook the op is the
// identity, which is what a single rank computes.
void set_all_reduce(std::function<void(void* data, size_t n, DType dtype)> hook);

// Worker threads for the parallel kernels (rayon's pool in rg). Results never depend on it.
void set_threads(int n);
int threads();

// Executes every step of `plan` over `slots`.
void exec_plan(const Plan& plan, std::vector<Buf>& slots);
// Fresh frame with constants loaded (plan.rs:641-647).
std::vector<Buf> frame(const Plan& plan);
// The given plan steps, in the given order, each as the interpreter runs it alone.
void exec_steps(const Plan& plan, const std::vector<size_t>& steps, std::vector<Buf>& slots);

// The CPU device: plans run in this interpreter.
std::shared_ptr<Device> cpu_device();
// Plans built with the CUDA device's fusion configuration and rewrites, run in this interpreter
// (device name "cuda-plan"; offered by `compile` but not listed as available).
std::shared_ptr<Device> cuda_plan_device();

}  // namespace rg::oracle
