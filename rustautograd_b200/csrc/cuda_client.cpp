// The product `_rg` module's device: every plan runs on the CUDA device through the C ABI of
// include/rgc.h (librgc_b200.so), exactly as an rg `src/cuda.rs` would drive it. There is no
// CPU execution path here: without a usable sm_100 GPU the device reports itself unavailable.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <stdexcept>

#include "blob.h"
#include "exec.h"
#include "rgc.h"

namespace py = pybind11;

namespace rg {

namespace {

[[noreturn]] void throw_rgc(const char* what) { throw std::runtime_error(std::string(what) + ": " + rgc_last_error()); }

class CudaExec : public Exec {
 public:
  CudaExec(rgc_program* p, const Plan& plan) : plan_(plan) {
    if (rgc_exec_acquire(p, &e_) != RGC_OK) throw_rgc("rgc_exec_acquire");
  }
  ~CudaExec() override { rgc_exec_release(e_); }
  void load(size_t k, const Tensor& t) override {
    size_t bytes = plan_.input_ns[k] * dtype_size(plan_.slots[plan_.input_slots[k]].first);
    if (rgc_exec_load(e_, k, t.data.data(), std::min(bytes, t.data.bytes())) != RGC_OK) throw_rgc("rgc_exec_load");
  }
  void step() override { last_ = rgc_exec_step(e_); }
  void step_at(size_t k) override { last_ = rgc_exec_step_at(e_, k); }
  void swap(size_t a, size_t b) override {
    if (rgc_exec_swap(e_, a, b) != RGC_OK) throw_rgc("rgc_exec_swap");
  }
  Buf prefix(size_t slot, size_t n) override {
    Buf b(plan_.slots[slot].first, n);
    if (rgc_exec_prefix(e_, slot, b.data(), b.bytes()) != RGC_OK) failed_read_ = rgc_last_error();
    return b;
  }
  void write_prefix(size_t slot, const Buf& b) override {
    if (rgc_exec_write_prefix(e_, slot, b.data(), b.bytes()) != RGC_OK) throw_rgc("rgc_exec_write_prefix");
  }
  double scalar(size_t slot) override {
    double v = 0;
    if (rgc_exec_scalar(e_, slot, &v) != RGC_OK) failed_read_ = rgc_last_error();
    return v;
  }
  std::optional<std::string> failure() override {
    char buf[1024];
    if (rgc_exec_failure(e_, buf, sizeof buf)) return std::string(buf);
    if (last_ != RGC_OK) return std::string(rgc_last_error());
    if (!failed_read_.empty()) return failed_read_;
    return std::nullopt;
  }
  bool run(const RunSpec& spec, const std::vector<const Tensor*>& state, const std::vector<std::vector<const Tensor*>>& batches,
           size_t steps, RunOut* out) override {
    std::vector<size_t> si, so;
    for (auto& [i, o] : spec.state) {
      si.push_back(i);
      so.push_back(o);
    }
    rgc_run_spec rs{si.data(), so.data(), si.size(), spec.data.data(), spec.data.size(), spec.history.data(), spec.history.size()};
    std::vector<const void*> st;
    for (const Tensor* t : state) st.push_back(t->data.data());
    const void* const* state_ptrs = spec.resident ? nullptr : st.data();
    std::vector<const void*> bt;
    for (auto& b : batches)
      for (size_t d = 0; d < spec.data.size(); ++d) bt.push_back(b[d]->data.data());
    std::vector<double> hist(spec.history.size() * steps);
    std::vector<Buf> outs;
    std::vector<void*> optr;
    std::vector<size_t> obytes;
    // State outputs get no host buffer here: they come back once, as the new state (below), and
    // the outputs hold empty placeholders for them (`state_outputs_elided`); a resident run
    // leaves the state on the device and its placeholders stay empty.
    std::vector<bool> is_state(plan_.outputs.size(), false);
    for (auto& [i, o] : spec.state) {
      (void)i;
      is_state[o] = true;
    }
    for (size_t o = 0; o < plan_.outputs.size(); ++o) outs.emplace_back(plan_.slots[plan_.outputs[o].slot].first, is_state[o] ? 0 : plan_.outputs[o].n);
    for (auto& b : outs) {
      optr.push_back(b.data());
      obytes.push_back(b.bytes());
    }
    size_t done = 0;
    int64_t bad = -1;
    double secs = 0;
    // State outputs come back through the state inputs (below), not a second copy.
    for (auto& [i, o] : spec.state) {
      (void)i;
      optr[o] = nullptr;
      obytes[o] = 0;
    }
    int rc = rgc_exec_run(e_, &rs, state_ptrs, bt.data(), batches.size(), steps, hist.data(), optr.data(), obytes.data(), &done, &bad, &secs);
    out->steps = done;
    out->seconds = secs;
    if (bad >= 0) out->nonfinite_step = (size_t)bad;
    if (rc != RGC_OK) out->device_error = std::string(rgc_last_error());
    out->history.assign(spec.history.size(), {});
    for (size_t h = 0; h < spec.history.size(); ++h) out->history[h].assign(hist.begin() + h * steps, hist.begin() + h * steps + done);
    if (!spec.resident) {
      for (auto& [i, o] : spec.state) {
        size_t slot = plan_.input_slots[i];
        Buf b(plan_.slots[slot].first, plan_.input_ns[i]);
        rgc_exec_prefix(e_, slot, b.data(), b.bytes());
        out->state.emplace_back(plan_.outputs[o].shape, std::move(b));
      }
      out->state_outputs_elided = done > 0;
    }
    if (done) {
      for (size_t o = 0; o < plan_.outputs.size(); ++o) {
        std::vector<size_t> shape = outs[o].n == 0 && is_state[o] ? std::vector<size_t>{0} : plan_.outputs[o].shape;
        out->outputs.emplace_back(shape, std::move(outs[o]));
      }
    }
    return true;
  }
  bool save_slots(const std::string& path, const std::string& header, const std::vector<size_t>& slots, const std::vector<size_t>& sizes) override {
    if (rgc_exec_save_slots(e_, path.c_str(), header.data(), header.size(), slots.data(), sizes.data(), slots.size()) != RGC_OK)
      throw std::runtime_error(rgc_last_error());
    return true;
  }
  bool load_slots(const std::string& path, const std::vector<uint64_t>& offsets, const std::vector<size_t>& slots, const std::vector<size_t>& sizes) override {
    if (rgc_exec_load_slots(e_, path.c_str(), offsets.data(), slots.data(), sizes.data(), slots.size()) != RGC_OK)
      throw std::runtime_error(rgc_last_error());
    return true;
  }
  rgc_exec* handle() { return e_; }

 private:
  const Plan& plan_;
  rgc_exec* e_ = nullptr;
  int last_ = RGC_OK;
  std::string failed_read_;
};

class CudaProgram : public Program {
 public:
  explicit CudaProgram(const Plan& plan) : plan_(plan) {
    auto blob = encode_plan(plan);
    if (rgc_program_create(blob.data(), blob.size(), -1, &p_) != RGC_OK) throw_rgc("the CUDA device could not build this plan");
  }
  ~CudaProgram() override { rgc_program_destroy(p_); }
  std::unique_ptr<Exec> exec() override { return std::make_unique<CudaExec>(p_, plan_); }
  size_t allocated_bytes() const override { return rgc_program_allocated_bytes(p_); }
  void inject_failure_for_test() override { rgc_program_inject_failure(p_); }
  bool step_checked(Exec& e, std::vector<int32_t>& flags) override {
    int rc = rgc_exec_step_checked(static_cast<CudaExec&>(e).handle(), flags.data(), flags.size());
    if (rc != RGC_OK) throw std::runtime_error(rgc_last_error());
    return true;
  }
  bool step_timed(Exec& e, std::vector<double>& seconds) override {
    return rgc_exec_step_timed(static_cast<CudaExec&>(e).handle(), seconds.data(), seconds.size()) == RGC_OK;
  }
  Json breakdown(Exec& e, size_t repeats) override {
    char buf[1024];
    if (rgc_exec_breakdown_json(static_cast<CudaExec&>(e).handle(), repeats, buf, sizeof buf) != RGC_OK) return Json();
    // The text is already JSON; carry it as a string field the caller can parse.
    Json j = Json::object();
    j["device"] = "cuda";
    j["raw"] = std::string(buf);
    return j;
  }
  uint64_t launches() const override { return rgc_program_launches(p_); }

 private:
  Plan plan_;
  rgc_program* p_ = nullptr;
};

class CudaDevice : public Device {
 public:
  std::string name() const override { return "cuda"; }
  bool available() const override { return rgc_available() == 1; }
  Fuse fuse() const override { return Fuse::CUDA(); }
  std::shared_ptr<Program> compile(const Plan& plan) override {
    if (!available()) throw std::runtime_error("no sm_100 CUDA device is available");
    auto p = std::make_shared<CudaProgram>(plan);
    programs_.push_back(p);
    return p;
  }
  uint64_t launches() {
    uint64_t n = 0;
    for (auto it = programs_.begin(); it != programs_.end();) {
      if (auto p = it->lock()) {
        n += p->launches();
        ++it;
      } else {
        it = programs_.erase(it);
      }
    }
    return n + retired_;
  }

 private:
  std::vector<std::weak_ptr<CudaProgram>> programs_;
  uint64_t retired_ = 0;
};

std::shared_ptr<CudaDevice> cuda() {
  static auto d = std::make_shared<CudaDevice>();
  return d;
}

}  // namespace

std::vector<std::string> module_available_devices() {
  if (cuda()->available()) return {"cuda"};
  return {};
}

std::shared_ptr<Device> module_device(const std::string& name) {
  if (name == "cuda" && cuda()->available()) return cuda();
  return nullptr;
}

void module_extra(py::module_& m) {
  // Constant folding and eager operations run on the device too.
  set_evaluator([](const Plan& p, const std::vector<const Tensor*>& in) {
    if (!cuda()->available()) throw std::runtime_error("no sm_100 CUDA device is available to evaluate on");
    return run_once(*cuda(), p, in);
  });
  m.def("cuda_available", [] { return rgc_available() == 1; });
  m.def("dist_unique_id", [] {
    uint8_t id[128];
    if (rgc_dist_unique_id(id) != RGC_OK) throw std::runtime_error("NCCL unavailable");
    return py::bytes((const char*)id, 128);
  });
  m.def("dist_init", [](int rank, int world, py::bytes id) {
    std::string_view v = id;
    if (v.size() != 128) throw py::value_error("NCCL unique id must be 128 bytes");
    if (rgc_dist_init(rank, world, (const uint8_t*)v.data()) != RGC_OK) throw std::runtime_error("NCCL communicator initialisation failed");
  });
  m.def("dist_finalize", [] { rgc_dist_finalize(); });
}

}  // namespace rg
