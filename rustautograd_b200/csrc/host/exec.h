// The device contract a plan executes through (restates plan.rs:29-41 `Exec` and the program /
// exec split of metal.rs:362-571). A `Device` turns a plan into a `Program` once, at compile
// time; a `Program` hands out `Exec` frames, one per call or run.
#pragma once
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "plan.h"

namespace rg {

// validate.rs:248-268
struct RunSpec {
  std::vector<std::pair<size_t, size_t>> state;  // (input index, output index) fed back each step
  std::vector<size_t> data;
  std::vector<size_t> history;  // scalar outputs recorded per step
  // The state already lives in the exec's state inputs (an earlier run, a load or a checkpoint
  // restore) and stays there afterwards: nothing is uploaded or read back.
  bool resident = false;
};

struct RunOut {
  std::vector<Tensor> state;
  std::vector<Tensor> outputs;
  std::vector<std::vector<double>> history;
  size_t steps = 0;
  std::optional<size_t> nonfinite_step;
  double seconds = 0;
  std::optional<std::string> device_error;
  // Set by a device run that returns state outputs only once, as `state`: outputs[o] of every
  // state pair (i, o) is then an empty placeholder whose value is the matching state tensor.
  bool state_outputs_elided = false;
};

struct Exec {
  virtual ~Exec() = default;
  virtual void load(size_t input, const Tensor& t) = 0;
  virtual void step() = 0;
  // Executes only step `k` of the plan: the instrumented (diagnostic) runs go one step at a time.
  virtual void step_at(size_t k) = 0;
  virtual void swap(size_t a, size_t b) = 0;
  virtual Buf prefix(size_t slot, size_t n) = 0;
  virtual void write_prefix(size_t slot, const Buf& b) = 0;
  virtual double scalar(size_t slot) = 0;
  virtual std::optional<std::string> failure() { return std::nullopt; }
  // Checkpoint streaming (checkpoint.py:37-105 layout) straight between slots and a file:
  // `header` then sizes[k] bytes of each slot, or file bytes at offsets[k] into each slot.
  // False where the device has no direct path (the caller then goes through prefix and
  // write_prefix).
  virtual bool save_slots(const std::string&, const std::string&, const std::vector<size_t>&, const std::vector<size_t>&) { return false; }
  virtual bool load_slots(const std::string&, const std::vector<uint64_t>&, const std::vector<size_t>&, const std::vector<size_t>&) { return false; }
  // A device-resident implementation of the whole multi-step loop. Returns false when the
  // device has none, and the host loop (run_loop) drives load/step/swap instead.
  // State and batch tensors are borrowed for the call (no host copies of them are made).
  virtual bool run(const RunSpec&, const std::vector<const Tensor*>&, const std::vector<std::vector<const Tensor*>>&, size_t, RunOut*) {
    return false;
  }
};

struct Program {
  virtual ~Program() = default;
  virtual std::unique_ptr<Exec> exec() = 0;
  virtual size_t allocated_bytes() const { return 0; }
  virtual void inject_failure_for_test() {}
  // Per-step timing and a launch breakdown for `profile` (metal.rs:692-712).
  virtual bool step_timed(Exec&, std::vector<double>&) { return false; }
  // One step with non-finite and index-range flags per plan step (2 x steps entries), computed
  // on the device; false where the device has no such scan.
  virtual bool step_checked(Exec&, std::vector<int32_t>&) { return false; }
  virtual Json breakdown(Exec&, size_t) { return Json(); }
  // Device kernels launched on behalf of this program so far (0 where not counted).
  virtual uint64_t launches() const { return 0; }
};

// Algorithmic work of each plan step: floating-point operations (2 per multiply-add) and the
// bytes a step must read and write at least once. The roofline of a kernel is judged on these.
struct StepCost {
  std::string kind;  // "fused", "matmul", "reduce", ... (the op name for single instructions)
  double flops = 0, bytes = 0;
};
std::vector<StepCost> step_costs(const Plan& p);

struct Device {
  virtual ~Device() = default;
  virtual std::string name() const = 0;
  virtual bool available() const = 0;
  // The fusion configuration plans for this device are built with.
  virtual Fuse fuse() const = 0;
  // Compile-time failures (kernel build, memory) throw std::runtime_error.
  virtual std::shared_ptr<Program> compile(const Plan& plan) = 0;
};

// Runs a plan once on a device with fresh buffers: the evaluator behind constant folding and
// eager operations.
std::vector<Tensor> run_once(Device& d, const Plan& plan, const std::vector<const Tensor*>& inputs);

// validate.rs:290-363, generic over the device.
RunOut run_loop(const Plan& p, Exec& e, const RunSpec& spec, const std::vector<Tensor>& state,
                const std::vector<std::vector<Tensor>>& batches, size_t steps);

}  // namespace rg
