// TEST INFRASTRUCTURE — the `_rg_oracle` Python module: rg's `_rg` interface over the CPU
// restatement of its interpreter (device "cpu"). Tests use it to drive rg's front end on the
// CPU, to pin the restatement against rg's golden vectors, and to execute plan blobs produced
// by the CUDA backend as the parity reference. bench.py times it as the CPU baseline.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "../rustautograd_b200/csrc/host/blob.h"
#include "../rustautograd_b200/csrc/host/validate.h"
#include "interp.h"

namespace py = pybind11;

namespace rg {

std::vector<std::string> module_available_devices() { return {"cpu"}; }

std::shared_ptr<Device> module_device(const std::string& name) {
  if (name == "cpu") return oracle::cpu_device();
  if (name == "cuda-plan") return oracle::cuda_plan_device();
  return nullptr;
}

void module_extra(py::module_& m) {
  set_evaluator([](const Plan& p, const std::vector<const Tensor*>& in) { return run_once(*oracle::cpu_device(), p, in); });
  m.def("set_threads", [](int n) { oracle::set_threads(n); });
  m.def("threads", [] { return oracle::threads(); });
  // Installs the cross-rank sum of the `all_reduce` op: fn(bytes, dtype) -> bytes of the sum.
  // Multi-process tests pass a torch.distributed (gloo) all-reduce here; None removes it.
  m.def("set_all_reduce", [](py::object fn) {
    if (fn.is_none()) {
      oracle::set_all_reduce(nullptr);
      return;
    }
    // The callable outlives this call; if it is still installed when the interpreter has shut
    // down, it is left alone rather than released without a live interpreter.
    auto keep = std::shared_ptr<py::object>(new py::object(fn), [](py::object* o) {
      if (Py_IsInitialized()) {
        py::gil_scoped_acquire gil;
        delete o;
      }
    });
    oracle::set_all_reduce([keep](void* data, size_t n, DType d) {
      py::gil_scoped_acquire gil;
      size_t bytes = n * dtype_size(d);
      py::bytes out = (*keep)(py::bytes((const char*)data, bytes), std::string(dtype_name(d)));
      std::string_view v = out;
      if (v.size() != bytes) throw std::runtime_error("all_reduce hook returned the wrong number of bytes");
      std::memcpy(data, v.data(), bytes);
    });
  });
  // Executes a plan blob (the C-ABI wire format) once on the CPU: inputs and outputs are
  // (bytes, shape, dtype) triples, so results cross between modules as plain data.
  m.def("run_plan_blob", [](py::bytes blob, std::vector<std::tuple<py::bytes, std::vector<size_t>, std::string>> inputs) {
    std::string_view b = blob;
    Plan p = decode_plan((const uint8_t*)b.data(), b.size());
    std::vector<Tensor> ts;
    for (auto& [data, shape, dtype] : inputs) {
      DType d;
      if (!parse_dtype(dtype, &d)) throw py::value_error("unsupported dtype " + dtype);
      std::string_view v = data;
      Buf buf(d, product(shape));
      if (v.size() != buf.bytes()) throw py::value_error("input bytes do not fit its shape");
      std::memcpy(buf.data(), v.data(), v.size());
      ts.emplace_back(shape, std::move(buf));
    }
    if (ts.size() != p.input_slots.size()) throw py::value_error("wrong number of inputs for this plan");
    std::vector<const Tensor*> ptrs;
    for (auto& t : ts) ptrs.push_back(&t);
    std::vector<Tensor> out;
    {
      py::gil_scoped_release nogil;
      out = run_once(*oracle::cpu_device(), p, ptrs);
    }
    py::list res;
    for (auto& t : out) res.append(py::make_tuple(py::bytes((const char*)t.data.data(), t.data.bytes()), t.shape, std::string(dtype_name(t.dtype()))));
    return res;
  });
  // Every slot of a plan blob's frame after loading `inputs` and running the plan steps listed in
  // `steps`, in that order: (bytes, dtype) per slot. Tests run a device kernel that stands for
  // some steps from the slots before them and compare with the slots after them.
  m.def("plan_blob_slots", [](py::bytes blob, std::vector<std::tuple<py::bytes, std::vector<size_t>, std::string>> inputs,
                              std::vector<size_t> steps) {
    std::string_view b = blob;
    Plan p = decode_plan((const uint8_t*)b.data(), b.size());
    if (inputs.size() != p.input_slots.size()) throw py::value_error("wrong number of inputs for this plan");
    auto slots = oracle::frame(p);
    for (size_t k = 0; k < inputs.size(); ++k) {
      std::string_view v = std::get<0>(inputs[k]);
      Buf& dst = slots[p.input_slots[k]];
      if (v.size() > dst.bytes()) throw py::value_error("input larger than its slot");
      std::memcpy(dst.data(), v.data(), v.size());
    }
    {
      py::gil_scoped_release nogil;
      oracle::exec_steps(p, steps, slots);
    }
    py::list res;
    for (auto& s : slots) res.append(py::make_tuple(py::bytes((const char*)s.data(), s.bytes()), std::string(dtype_name(s.dtype))));
    return res;
  });
  // Multi-step run of a plan blob on the CPU with rg's run-loop semantics, for history parity.
  m.def("run_plan_blob_steps", [](py::bytes blob, std::vector<std::pair<size_t, size_t>> state_map, std::vector<size_t> data_inputs,
                                  std::vector<size_t> history, std::vector<std::tuple<py::bytes, std::vector<size_t>, std::string>> inputs, size_t steps) {
    std::string_view b = blob;
    Plan p = decode_plan((const uint8_t*)b.data(), b.size());
    auto to_tensor = [](const std::tuple<py::bytes, std::vector<size_t>, std::string>& x) {
      DType d;
      if (!parse_dtype(std::get<2>(x), &d)) throw py::value_error("unsupported dtype");
      std::string_view v = std::get<0>(x);
      Buf buf(d, product(std::get<1>(x)));
      if (v.size() != buf.bytes()) throw py::value_error("input bytes do not fit its shape");
      std::memcpy(buf.data(), v.data(), v.size());
      return Tensor(std::get<1>(x), std::move(buf));
    };
    RunSpec spec{state_map, data_inputs, history};
    std::vector<Tensor> state;
    std::vector<Tensor> batch;
    for (size_t k = 0; k < inputs.size(); ++k) (k < state_map.size() ? state : batch).push_back(to_tensor(inputs[k]));
    std::vector<std::vector<Tensor>> batches;
    if (!batch.empty()) batches.push_back(batch);
    RunOut out;
    {
      py::gil_scoped_release nogil;
      auto prog = oracle::cpu_device()->compile(p);
      auto e = prog->exec();
      out = run_loop(p, *e, spec, state, batches, steps);
    }
    py::list st;
    for (auto& t : out.state) st.append(py::make_tuple(py::bytes((const char*)t.data.data(), t.data.bytes()), t.shape, std::string(dtype_name(t.dtype()))));
    return py::make_tuple(st, out.history, out.steps, out.seconds);
  });
}

}  // namespace rg
