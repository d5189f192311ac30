// Compiled programs: build, validate, call, run (restates src/validate.rs).
#pragma once
#include <functional>
#include <memory>
#include <mutex>

#include "exec.h"
#include "optimize.h"

namespace rg {

enum class Level { None = 0, Basic = 1, Standard = 2, Thorough = 3 };
bool parse_level(const std::string& s, Level* l);

// Runs a plan on the CPU reference interpreter, when the embedding process provides one; the
// device-equivalence check (validate.rs:674-705) compares against it.
using ReferenceRunner = std::function<std::vector<Tensor>(const Plan&, const std::vector<Tensor>&)>;
void set_reference_runner(ReferenceRunner r);

Json device_failure(const std::string& device, const std::string& error);

class Compiled {
 public:
  Graph raw;
  std::vector<uint32_t> outputs;
  Plan plan;
  Plan raw_plan;
  Json report;
  Level level = Level::None;
  std::shared_ptr<Device> device;
  std::shared_ptr<Program> program;
  OptMode mode = OptMode::Standard;
  OptStats opt_stats;

  void check_inputs(const std::vector<Tensor>& inputs) const;
  std::vector<Tensor> try_call(const std::vector<Tensor>& inputs) const;  // throws DiagError
  Json check(const std::vector<Tensor>& inputs) const;
  Json profile(const std::vector<Tensor>& inputs, size_t repeats) const;
  void validate_spec(const RunSpec& spec) const;
  RunOut run(const RunSpec& spec, const std::vector<Tensor>& state, const std::vector<std::vector<Tensor>>& batches, size_t steps) const;
  // The same run over borrowed tensors; the result may have `state_outputs_elided` set.
  RunOut run_refs(const RunSpec& spec, const std::vector<const Tensor*>& state, const std::vector<std::vector<const Tensor*>>& batches,
                  size_t steps) const;
  // (step, batch index, state before it) of the first non-finite step, if any.
  bool replay(const RunSpec& spec, const std::vector<Tensor>& state, const std::vector<std::vector<Tensor>>& batches, size_t steps,
              size_t* step, size_t* batch, std::vector<Tensor>* before) const;

  // Internal pieces of validation, public for the builder below.
  Json validate(const std::vector<Tensor>& examples);

 private:
  struct Observed {
    std::vector<Json> roots, hard;
    size_t propagated = 0;
    std::vector<Tensor> values;
  };
  Observed observed(const std::vector<Tensor>& inputs) const;
  // The observer's common case on a device with a per-step scan: the optimised plan of all
  // outputs and gradients run once with non-finite and index flags computed on the device.
  // Returns the values when nothing was flagged (nothing to explain), else nothing.
  std::optional<std::vector<Tensor>> scanned(const std::vector<Tensor>& inputs) const;
  std::vector<uint32_t> raw_outputs() const;
  std::pair<Json, std::vector<Json>> gradient_stats(const std::vector<Tensor>& vals) const;
  Json optimizer_check(const std::vector<Tensor>& examples) const;  // throws DiagError
  std::pair<Json, std::vector<Json>> device_check(const std::vector<Tensor>& examples) const;
  std::pair<Json, std::vector<Json>> grad_check(const std::vector<Tensor>& examples) const;
  std::pair<Json, std::vector<Json>> perturbation_check(const std::vector<Tensor>& examples) const;
  mutable std::shared_ptr<Program> raw_program_;
  mutable std::shared_ptr<Program> scan_program_;
  mutable Plan scan_plan_;
  mutable std::mutex mu_;
};

std::unique_ptr<Compiled> compile_mode(Graph raw, std::vector<uint32_t> outputs, const std::vector<Tensor>& examples, Level level,
                                       std::shared_ptr<Device> device, OptMode mode);

}  // namespace rg
