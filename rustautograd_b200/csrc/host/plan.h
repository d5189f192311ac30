// The executable step plan: scheduling, fusion groups and slot allocation (restates
// src/plan.rs:12-164 and 184-655). A plan is data: the host builds it, serialises it
// (blob.cpp) and a device executes it through the Exec contract (plan.rs:29-41).
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "graph.h"

namespace rg {

// plan.rs:12-27. `gpu` is rg's `metal` flag generalised: group chains of any cost, allow
// arbitrary broadcast inputs in groups, float only. `hoist` keeps the Metal behaviour of
// scheduling CPU-cheap work first; the CUDA device runs everything itself, so it is off there.
struct Fuse {
  double parallel_ns = 200000.0;
  bool gpu = false;
  bool levels = false;
  bool hoist = false;
  size_t max_bindings = 28;
  // Schedule tiny (at most 64-element) elementwise chains that depend only on inputs first, so
  // that a scalar chain (an optimizer's step count and bias corrections) does not push the
  // tensor ops that read it into a later dependency level and split their fusion group.
  bool hoist_small = false;
  // Level order only: an elementwise node whose every consumer is an elementwise node of its
  // shape and dtype moves up to the level of its first consumer, so that it runs inside that
  // consumer's group. A value recomputed for the backward pass (a rematerialisation clone) then
  // fuses into the backward group that reads it instead of being written by the forward group.
  bool sink = false;

  static Fuse DEFAULT() { return Fuse{200000.0, false, false, false, 28, false, false}; }
  static Fuse METAL() { return Fuse{0.0, true, true, true, 28, false, false}; }
  // The CUDA device's configuration: groups of any cost, in dependency-level order when that
  // is cheaper, with up to 64 bindings per kernel (kernel parameters, not a binding table).
  static Fuse CUDA() { return Fuse{0.0, true, true, false, 64, true, true}; }
  std::string key() const {
    return std::to_string(parallel_ns) + (gpu ? "g" : "c") + (levels ? "l" : "n") + (hoist ? "h" : "x") + std::to_string(max_bindings) +
           (hoist_small ? "s" : "") + (sink ? "k" : "");
  }
};

enum class ArgKind : uint8_t { Full = 0, Splat = 1, Row = 2, Broadcast = 3 };

struct Operand {
  bool reg = false;  // false: full input k; true: register r
  size_t idx = 0;
};

struct MicroOp {
  Op op;
  size_t reg = 0;
  std::vector<Operand> args;
};

struct FusedInput {
  size_t slot = 0;
  ArgKind kind = ArgKind::Full;
  size_t row = 0;  // Row(L)
  size_t reg = SIZE_MAX;
};

struct Fused {
  DType dtype = DType::F32;
  size_t n = 0;
  std::vector<FusedInput> inputs;
  std::vector<MicroOp> ops;
  std::vector<std::pair<size_t, size_t>> outputs;  // (register, slot); never aliases an input
  size_t regs = 0;
  std::vector<size_t> shape;
  std::vector<std::vector<size_t>> input_shapes;
};

enum class Mode : uint8_t { Same = 0, AScalar = 1, BScalar = 2, General = 3 };

struct Instr {
  Op op;
  uint32_t node = 0;
  DType dtype = DType::F32;
  size_t dst = SIZE_MAX;
  std::vector<size_t> args;
  std::vector<size_t> shape;
  std::vector<std::vector<size_t>> arg_shapes;
  size_t n = 0;
  Mode mode = Mode::Same;
  std::vector<std::pair<size_t, size_t>> outs;  // control flow: (output index, slot)
  // Control flow: the plans its bodies execute (Scan body / While cond, body / Cond then, else).
  std::shared_ptr<Plan> body_plan, body2_plan;
};

struct Step {
  bool fused = false;
  Instr instr;
  Fused group;
};

struct PlanOutput {
  size_t slot = 0;
  std::vector<size_t> shape;
  size_t n = 0;
};

struct Plan {
  std::vector<Step> steps;
  std::vector<std::pair<DType, size_t>> slots;
  std::vector<bool> pinned;
  std::vector<std::pair<size_t, TensorP>> consts;
  std::vector<size_t> input_slots;
  std::vector<size_t> input_ns;
  std::vector<PlanOutput> outputs;
  bool reference = false;
  size_t naive_bytes = 0;
  size_t peak_live_bytes = 0;
  // The fusion configuration control-flow bodies are built with (their plans are nested).
  Fuse fuse = Fuse::DEFAULT();

  static Plan build(const Graph& g, const std::vector<uint32_t>& outputs, bool reuse);
  static Plan build_fused(const Graph& g, const std::vector<uint32_t>& outputs, const Fuse& cfg);
  double gpu_cost_estimate() const;
  size_t planned_bytes() const;
  size_t n_fused() const;
  size_t n_fused_ops() const;

 private:
  static Plan build_with(const Graph& g, const std::vector<uint32_t>& outputs, bool reuse, const Fuse* fuse);
};

// Helpers shared by the executors.
std::vector<size_t> strides(const std::vector<size_t>& shape);
std::vector<size_t> bstrides(const std::vector<size_t>& shape, size_t rank);
Mode binary_mode(const Op& op, const std::vector<size_t>& shape, const std::vector<std::vector<size_t>>& args);
bool is_alias(const Graph& g, size_t id);

// One-off evaluation of a graph (plan.rs:1023-1032 `eval`). The host compiler needs it for
// constant folding and the front end for eager operations; the executing device is whatever the
// embedding module installs (the CUDA device in the product module).
using EvalFn = std::function<std::vector<Tensor>(const Plan&, const std::vector<const Tensor*>&)>;
void set_evaluator(EvalFn f);
bool has_evaluator();
std::vector<Tensor> eval(const Graph& g, const std::vector<uint32_t>& outputs, const std::vector<const Tensor*>& inputs);

}  // namespace rg
