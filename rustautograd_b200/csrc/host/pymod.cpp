// The `_rg` Python module: the same classes, methods and error behaviour as rg's PyO3 module
// (src/python.rs:12-303), so rg's own Python front end, or this package's, drives the engine.
// The devices it offers come from the build it is linked into (module_devices below).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "autodiff.h"
#include "blob.h"
#include "rowchain.h"
#include "validate.h"

namespace py = pybind11;

namespace rg {
// Provided by the build this module is linked into.
std::vector<std::string> module_available_devices();
std::shared_ptr<Device> module_device(const std::string& name);
void module_extra(py::module_& m);
}  // namespace rg

using namespace rg;

namespace {

py::object g_diag_type;

[[noreturn]] void raise_diag(const Json& d) {
  std::string text = d.dump();
  py::object err = g_diag_type(text);
  try {
    err.attr("diagnostic") = py::module_::import("json").attr("loads")(text);
  } catch (...) {
  }
  PyErr_SetObject(g_diag_type.ptr(), err.ptr());
  throw py::error_already_set();
}

DType dtype_arg(const std::string& s) {
  DType d;
  if (!parse_dtype(s, &d)) throw py::value_error("unsupported dtype " + s);
  return d;
}

struct PyTensor {
  std::shared_ptr<const Tensor> t;
};

PyTensor make_tensor(py::bytes data, std::vector<size_t> shape, const std::string& dtype) {
  DType d = dtype_arg(dtype);
  std::string_view view = data;
  size_t n = product(shape);
  if (view.size() != n * dtype_size(d))
    throw py::value_error(std::to_string(view.size()) + " bytes do not fit shape " + Json(shape).dump() + " of " + dtype_name(d));
  Buf b(d, n);
  std::memcpy(b.data(), view.data(), view.size());
  return PyTensor{std::make_shared<const Tensor>(std::move(shape), std::move(b))};
}

std::vector<Tensor> tensors(const std::vector<PyTensor>& v) {
  std::vector<Tensor> out;
  out.reserve(v.size());
  for (auto& p : v) out.push_back(*p.t);
  return out;
}

// Borrowed views of Python-held tensors (immutable, kept alive by the caller's list).
std::vector<const Tensor*> refs(const std::vector<PyTensor>& v) {
  std::vector<const Tensor*> out;
  out.reserve(v.size());
  for (auto& p : v) out.push_back(p.t.get());
  return out;
}

std::vector<PyTensor> wrap(std::vector<Tensor> v) {
  std::vector<PyTensor> out;
  for (auto& t : v) out.push_back(PyTensor{std::make_shared<const Tensor>(std::move(t))});
  return out;
}

template <typename T> T attr(const py::dict* a, const char* key) {
  if (!a || !a->contains(key)) throw py::value_error(std::string("missing attribute ") + key);
  try {
    return (*a)[key].cast<T>();
  } catch (const py::cast_error&) {
    throw py::value_error(std::string("invalid attribute ") + key);
  }
}

// python.rs:88-133
Op parse_op(const std::string& name, const py::dict* a) {
  auto reduce = [&](ReduceKind k) {
    Op o = Op::make(OpKind::Reduce);
    o.reduce = k;
    o.shape = attr<std::vector<size_t>>(a, "axes");
    o.flag_a = attr<bool>(a, "keepdims");
    return o;
  };
  static const std::pair<const char*, OpKind> simple[] = {
      {"neg", OpKind::Neg}, {"exp", OpKind::Exp}, {"log", OpKind::Log}, {"sqrt", OpKind::Sqrt}, {"sin", OpKind::Sin},
      {"cos", OpKind::Cos}, {"tanh", OpKind::Tanh}, {"abs", OpKind::Abs}, {"sign", OpKind::Sign}, {"add", OpKind::Add},
      {"sub", OpKind::Sub}, {"mul", OpKind::Mul}, {"div", OpKind::Div}, {"pow", OpKind::Pow}, {"maximum", OpKind::Max},
      {"minimum", OpKind::Min}, {"gt", OpKind::Gt}, {"ge", OpKind::Ge}, {"where", OpKind::Where}, {"matmul", OpKind::MatMul},
      {"stop_gradient", OpKind::StopGradient}, {"floor", OpKind::Floor}, {"take_along", OpKind::TakeAlong}, {"argmax", OpKind::Argmax}, {"all_reduce", OpKind::AllReduce},
  };
  for (auto& [n, k] : simple)
    if (name == n) return Op::make(k);
  if (name == "sum") return reduce(ReduceKind::Sum);
  if (name == "max") return reduce(ReduceKind::Max);
  if (name == "min") return reduce(ReduceKind::Min);
  Op o;
  if (name == "reshape") { o.kind = OpKind::Reshape; o.shape = attr<std::vector<size_t>>(a, "shape"); return o; }
  if (name == "transpose") { o.kind = OpKind::Transpose; o.shape = attr<std::vector<size_t>>(a, "perm"); return o; }
  if (name == "broadcast_to") { o.kind = OpKind::BroadcastTo; o.shape = attr<std::vector<size_t>>(a, "shape"); return o; }
  if (name == "slice") {
    o.kind = OpKind::Slice;
    o.starts = attr<std::vector<size_t>>(a, "starts");
    o.stops = attr<std::vector<size_t>>(a, "stops");
    return o;
  }
  if (name == "cast") { o.kind = OpKind::Cast; o.dtype = dtype_arg(attr<std::string>(a, "dtype")); return o; }
  if (name == "take") { o.kind = OpKind::Take; o.index = attr<size_t>(a, "axis"); return o; }
  if (name == "concat") { o.kind = OpKind::Concat; o.index = attr<size_t>(a, "axis"); return o; }
  if (name == "arg_top_k") { o.kind = OpKind::ArgTopK; o.index = attr<size_t>(a, "k"); return o; }
  if (name == "cumsum") { o.kind = OpKind::Cumsum; o.flag_a = attr<bool>(a, "reverse"); return o; }
  if (name == "random_uniform" || name == "random_normal") {
    o.kind = name == "random_uniform" ? OpKind::RandUniform : OpKind::RandNormal;
    o.shape = attr<std::vector<size_t>>(a, "shape");
    o.dtype = dtype_arg(attr<std::string>(a, "dtype"));
    return o;
  }
  if (name == "key_split") { o.kind = OpKind::KeySplit; o.index = attr<size_t>(a, "n"); return o; }
  throw py::value_error("unknown op " + name);
}

std::shared_ptr<const std::string> src(const std::optional<std::string>& s) {
  return s ? std::make_shared<const std::string>(*s) : nullptr;
}

struct PyGraph {
  Graph g;
  void check_id(uint32_t id) const {
    if (id >= g.nodes.size()) throw py::index_error("unknown node id " + std::to_string(id));
  }
};

template <typename F> auto guarded(F f) -> decltype(f()) {
  try {
    return f();
  } catch (const DiagError& d) {
    raise_diag(d.diag);
  }
}

struct PyCompiled {
  std::unique_ptr<Compiled> c;
};

// Not in rg's module: a run whose state stays in one exec's frame between calls (on the CUDA
// device: in HBM), with checkpoints streamed between that frame and safetensors files.
struct PySession {
  py::object owner;  // the Compiled, kept alive
  const Compiled* c = nullptr;
  std::unique_ptr<Exec> e;
  RunSpec spec;
  bool resident = true;             // the device runs the loop itself
  std::vector<Tensor> host_state;   // otherwise the state between runs
  std::vector<size_t> state_slots() const {
    std::vector<size_t> v;
    for (auto& [i, o] : spec.state) v.push_back(c->plan.input_slots[i]);
    return v;
  }
  std::vector<size_t> state_bytes() const {
    std::vector<size_t> v;
    for (auto& [i, o] : spec.state) v.push_back(c->plan.input_ns[i] * dtype_size(c->plan.slots[c->plan.input_slots[i]].first));
    return v;
  }
};

}  // namespace

PYBIND11_MODULE(RG_MODULE_NAME, m) {
  m.doc() = "rg engine: graph IR, autodiff, optimiser, planner and device execution";
  g_diag_type = py::reinterpret_borrow<py::object>(PyErr_NewException((std::string(PYBIND11_TOSTRING(RG_MODULE_NAME)) + ".DiagnosticError").c_str(), PyExc_Exception, nullptr));
  m.attr("DiagnosticError") = g_diag_type;

  py::class_<PyTensor>(m, "Tensor")
      .def(py::init(&make_tensor), py::arg("data"), py::arg("shape"), py::arg("dtype"))
      .def_property_readonly("shape", [](const PyTensor& t) { return t.t->shape; })
      .def_property_readonly("dtype", [](const PyTensor& t) { return std::string(dtype_name(t.t->dtype())); })
      .def("is_finite", [](const PyTensor& t) { return t.t->is_finite(); })
      .def("tobytes", [](const PyTensor& t) { return py::bytes((const char*)t.t->data.data(), t.t->data.bytes()); });

  py::class_<PyGraph>(m, "Graph")
      .def(py::init<>())
      .def("input", [](PyGraph& self, std::vector<size_t> shape, const std::string& dtype, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return self.g.input(shape, dtype_arg(dtype));
          }, py::arg("shape"), py::arg("dtype"), py::arg("source") = py::none())
      .def("constant", [](PyGraph& self, const PyTensor& t, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return self.g.constant(t.t);
          }, py::arg("t"), py::arg("source") = py::none())
      .def("op", [](PyGraph& self, const std::string& name, std::vector<uint32_t> inputs, std::optional<py::dict> attrs, std::optional<std::string> source) {
            Op op = parse_op(name, attrs ? &*attrs : nullptr);
            self.g.cur_source = src(source);
            return guarded([&] { return self.g.add(std::move(op), inputs); });
          }, py::arg("name"), py::arg("inputs"), py::arg("attrs") = py::none(), py::arg("source") = py::none())
      .def("grad", [](PyGraph& self, uint32_t y, std::vector<uint32_t> wrts, std::optional<std::string> source) {
            self.check_id(y);
            for (auto w : wrts) self.check_id(w);
            self.g.cur_source = src(source);
            return guarded([&] { return grad(self.g, y, wrts); });
          }, py::arg("y"), py::arg("wrts"), py::arg("source") = py::none())
      .def("scan", [](PyGraph& self, const PyGraph& body, std::vector<uint32_t> outputs, size_t n_carry, size_t n_x, size_t length,
                      std::vector<uint32_t> inputs, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return guarded([&] {
              Op o = Op::make(OpKind::Scan);
              o.body = Body::make(body.g, outputs);
              o.n_carry = n_carry;
              o.n_x = n_x;
              o.length = length;
              return self.g.add(std::move(o), inputs);
            });
          }, py::arg("body"), py::arg("outputs"), py::arg("n_carry"), py::arg("n_x"), py::arg("length"), py::arg("inputs"), py::arg("source") = py::none())
      .def("while_loop", [](PyGraph& self, const PyGraph& cond, uint32_t cond_output, const PyGraph& body, std::vector<uint32_t> outputs,
                            size_t n_carry, size_t max_iterations, std::vector<uint32_t> inputs, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return guarded([&] {
              Op o = Op::make(OpKind::While);
              o.body = Body::make(cond.g, {cond_output});
              o.body2 = Body::make(body.g, outputs);
              o.n_carry = n_carry;
              o.max_iterations = max_iterations;
              return self.g.add(std::move(o), inputs);
            });
          }, py::arg("cond"), py::arg("cond_output"), py::arg("body"), py::arg("outputs"), py::arg("n_carry"), py::arg("max_iterations"),
          py::arg("inputs"), py::arg("source") = py::none())
      .def("cond", [](PyGraph& self, const PyGraph& then_body, std::vector<uint32_t> then_outputs, const PyGraph& else_body,
                      std::vector<uint32_t> else_outputs, std::vector<uint32_t> inputs, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return guarded([&] {
              Op o = Op::make(OpKind::Cond);
              o.body = Body::make(then_body.g, then_outputs);
              o.body2 = Body::make(else_body.g, else_outputs);
              return self.g.add(std::move(o), inputs);
            });
          }, py::arg("then_body"), py::arg("then_outputs"), py::arg("else_body"), py::arg("else_outputs"), py::arg("inputs"), py::arg("source") = py::none())
      .def("output", [](PyGraph& self, uint32_t node, size_t index, std::vector<size_t> shape, const std::string& dtype) {
            DType d = dtype_arg(dtype);
            Op o = Op::make(OpKind::Output);
            o.index = index;
            o.shape = shape;
            o.dtype = d;
            try {
              return self.g.add(std::move(o), {node});
            } catch (const DiagError&) {
              throw py::value_error("invalid control-flow output");
            }
          })
      .def("placeholder", [](PyGraph& self, std::vector<size_t> shape, const std::string& dtype) { return self.g.placeholder(shape, dtype_arg(dtype)); })
      .def("custom", [](PyGraph& self, uint32_t y, uint32_t placeholder, std::vector<std::pair<uint32_t, uint32_t>> rules, std::optional<std::string> source) {
            self.g.cur_source = src(source);
            return guarded([&] {
              Op o = Op::make(OpKind::Custom);
              o.placeholder = placeholder;
              o.rules = rules;
              return self.g.add(std::move(o), {y});
            });
          }, py::arg("y"), py::arg("placeholder"), py::arg("rules"), py::arg("source") = py::none())
      .def("grad_records", [](const PyGraph& self) {
        std::vector<std::tuple<uint32_t, uint32_t, uint32_t>> out;
        for (auto& r : self.g.grads) out.emplace_back(r.y, r.wrt, r.grad);
        return out;
      })
      .def("shape", [](const PyGraph& self, uint32_t id) {
        self.check_id(id);
        return self.g.shape(id);
      })
      .def("dtype", [](const PyGraph& self, uint32_t id) {
        self.check_id(id);
        return std::string(dtype_name(self.g.dtype(id)));
      })
      .def("eval", [](const PyGraph& self, std::vector<uint32_t> ids) {
        for (auto id : ids) self.check_id(id);
        std::vector<Tensor> out;
        {
          py::gil_scoped_release nogil;
          out = eval(self.g, ids, {});
        }
        return wrap(std::move(out));
      })
      // Not in rg's module: a description of the nodes, for tests that compare graphs.
      .def("_describe", [](const PyGraph& self) {
        Json a = Json::array();
        for (auto& n : self.g.nodes) {
          Json j = Json::object();
          j["op"] = n.op.name();
          j["key"] = n.op.key();
          j["inputs"] = Json(std::vector<size_t>(n.inputs.begin(), n.inputs.end()));
          j["shape"] = Json(n.shape);
          j["dtype"] = dtype_name(n.dtype);
          a.push(j);
        }
        return a.dump();
      })
      .def_property_readonly("n_nodes", [](const PyGraph& self) { return self.g.nodes.size(); });

  py::class_<PySession>(m, "Session")
      .def("run", [](PySession& self, std::vector<std::vector<PyTensor>> batches, size_t steps) {
        std::vector<std::vector<const Tensor*>> bs;
        for (auto& b : batches) bs.push_back(refs(b));
        RunOut out;
        {
          py::gil_scoped_release nogil;
          if (self.resident) {
            RunSpec spec = self.spec;
            spec.resident = true;
            self.resident = self.e->run(spec, {}, bs, steps, &out);
          }
          if (!self.resident) {
            std::vector<std::vector<Tensor>> owned;
            for (auto& b : batches) owned.push_back(tensors(b));
            out = run_loop(self.c->plan, *self.e, self.spec, self.host_state, owned, steps);
            self.host_state = out.state;
          }
        }
        if (out.device_error) {
          Json d = device_failure(self.c->device->name(), *out.device_error);
          d["observation"]["completed_steps"] = out.steps;
          raise_diag(d);
        }
        std::optional<size_t> bad = out.nonfinite_step;
        return py::make_tuple(wrap(std::move(out.outputs)), out.history, out.steps, bad, out.seconds);
      })
      .def("state", [](PySession& self) {
        if (!self.resident) return wrap(self.host_state);
        std::vector<Tensor> out;
        auto slots = self.state_slots();
        for (size_t k = 0; k < slots.size(); ++k) {
          auto [i, o] = self.spec.state[k];
          out.emplace_back(self.c->plan.outputs[o].shape, self.e->prefix(slots[k], self.c->plan.input_ns[i]));
        }
        return wrap(std::move(out));
      })
      .def("save", [](PySession& self, const std::string& path, py::bytes header) {
        std::string h = header;
        py::gil_scoped_release nogil;
        auto slots = self.state_slots();
        auto sizes = self.state_bytes();
        if (self.resident && self.e->save_slots(path, h, slots, sizes)) return;
        // Generic path: the state as host tensors, written in the same layout.
        std::string tmp = path + ".tmp";
        FILE* fp = std::fopen(tmp.c_str(), "wb");
        if (!fp) throw std::runtime_error("cannot open " + tmp + " for writing");
        uint64_t len = h.size();
        unsigned char le[8];
        for (int i = 0; i < 8; ++i) le[i] = (unsigned char)(len >> (8 * i));
        bool ok = std::fwrite(le, 1, 8, fp) == 8 && std::fwrite(h.data(), 1, h.size(), fp) == h.size();
        for (size_t k = 0; k < slots.size() && ok; ++k) {
          auto [i, o] = self.spec.state[k];
          (void)o;
          Buf b = self.resident ? self.e->prefix(slots[k], self.c->plan.input_ns[i]) : self.host_state[k].data;
          ok = std::fwrite(b.data(), 1, b.bytes(), fp) == b.bytes();
        }
        ok = (std::fclose(fp) == 0) && ok;
        if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("writing the checkpoint " + path + " failed");
      })
      .def("restore", [](PySession& self, const std::string& path, std::vector<uint64_t> offsets) {
        py::gil_scoped_release nogil;
        auto slots = self.state_slots();
        auto sizes = self.state_bytes();
        if (offsets.size() != slots.size()) throw std::runtime_error("one file offset per state tensor is needed");
        if (self.resident && self.e->load_slots(path, offsets, slots, sizes)) return;
        FILE* fp = std::fopen(path.c_str(), "rb");
        if (!fp) throw std::runtime_error("cannot open " + path);
        for (size_t k = 0; k < slots.size(); ++k) {
          auto [i, o] = self.spec.state[k];
          Buf b(self.c->plan.slots[slots[k]].first, self.c->plan.input_ns[i]);
          bool ok = std::fseek(fp, (long)offsets[k], SEEK_SET) == 0 && std::fread(b.data(), 1, b.bytes(), fp) == b.bytes();
          if (!ok) {
            std::fclose(fp);
            throw std::runtime_error(path + ": file shorter than its header says");
          }
          // Both copies: a device without a resident run loop uses the host copy.
          self.e->write_prefix(slots[k], b);
          self.host_state[k] = Tensor(self.c->plan.outputs[o].shape, std::move(b));
        }
        std::fclose(fp);
      });

  py::class_<PyCompiled>(m, "Compiled")
      .def("session", [](py::object owner, std::vector<std::pair<size_t, size_t>> state_map, std::vector<size_t> data_inputs,
                         std::vector<size_t> history, std::vector<PyTensor> state) {
        const PyCompiled& self = owner.cast<const PyCompiled&>();
        RunSpec spec{state_map, data_inputs, history};
        guarded([&] {
          self.c->validate_spec(spec);
          return 0;
        });
        PySession ses;
        ses.owner = owner;
        ses.c = self.c.get();
        ses.spec = spec;
        ses.host_state = tensors(state);
        {
          py::gil_scoped_release nogil;
          ses.e = self.c->program->exec();
          for (size_t k = 0; k < spec.state.size() && k < ses.host_state.size(); ++k) ses.e->load(spec.state[k].first, ses.host_state[k]);
        }
        return ses;
      })
      .def_property_readonly("report_json", [](const PyCompiled& self) { return self.c->report.dump(); })
      .def_property_readonly("output_shapes", [](const PyCompiled& self) {
        std::vector<std::vector<size_t>> s;
        for (auto& o : self.c->plan.outputs) s.push_back(o.shape);
        return s;
      })
      .def("call", [](const PyCompiled& self, std::vector<PyTensor> inputs) {
        auto in = tensors(inputs);
        return guarded([&] {
          self.c->check_inputs(in);
          std::vector<Tensor> out;
          {
            py::gil_scoped_release nogil;
            out = self.c->try_call(in);
          }
          return wrap(std::move(out));
        });
      })
      .def("check", [](const PyCompiled& self, std::vector<PyTensor> inputs) {
        auto in = tensors(inputs);
        return guarded([&] {
          self.c->check_inputs(in);
          py::gil_scoped_release nogil;
          return self.c->check(in).dump();
        });
      })
      .def("profile", [](const PyCompiled& self, std::vector<PyTensor> inputs, size_t repeats) {
        auto in = tensors(inputs);
        return guarded([&] {
          self.c->check_inputs(in);
          py::gil_scoped_release nogil;
          return self.c->profile(in, repeats).dump();
        });
      })
      .def("run", [](const PyCompiled& self, std::vector<std::pair<size_t, size_t>> state_map, std::vector<size_t> data_inputs,
                     std::vector<size_t> history, std::vector<PyTensor> state, std::vector<std::vector<PyTensor>> batches, size_t steps) {
        RunSpec spec{state_map, data_inputs, history};
        guarded([&] {
          self.c->validate_spec(spec);
          return 0;
        });
        auto st = refs(state);
        std::vector<std::vector<const Tensor*>> bs;
        for (auto& b : batches) bs.push_back(refs(b));
        RunOut out;
        {
          py::gil_scoped_release nogil;
          out = self.c->run_refs(spec, st, bs, steps);
        }
        if (out.device_error) {
          Json d = device_failure(self.c->device->name(), *out.device_error);
          d["observation"]["completed_steps"] = out.steps;
          raise_diag(d);
        }
        std::optional<size_t> bad = out.nonfinite_step;
        auto new_state = wrap(std::move(out.state));
        auto outputs = wrap(std::move(out.outputs));
        // A state output's value is the new state tensor: share it rather than copy it.
        if (out.state_outputs_elided)
          for (size_t k = 0; k < state_map.size() && k < new_state.size(); ++k)
            if (state_map[k].second < outputs.size()) outputs[state_map[k].second] = new_state[k];
        return py::make_tuple(new_state, outputs, out.history, out.steps, bad, out.seconds);
      })
      .def("replay", [](const PyCompiled& self, std::vector<std::pair<size_t, size_t>> state_map, std::vector<size_t> data_inputs,
                        std::vector<size_t> history, std::vector<PyTensor> state, std::vector<std::vector<PyTensor>> batches, size_t steps) -> py::object {
        RunSpec spec{state_map, data_inputs, history};
        auto st = tensors(state);
        std::vector<std::vector<Tensor>> bs;
        for (auto& b : batches) bs.push_back(tensors(b));
        size_t k = 0, b = 0;
        std::vector<Tensor> before;
        bool found;
        {
          py::gil_scoped_release nogil;
          found = self.c->replay(spec, st, bs, steps, &k, &b, &before);
        }
        if (!found) return py::none();
        return py::make_tuple(k, b, wrap(std::move(before)));
      })
      // Not in rg's module: the executed plan in the C-ABI wire format, for parity tests.
      .def("plan_blob", [](const PyCompiled& self) {
        auto b = encode_plan(self.c->plan);
        return py::bytes((const char*)b.data(), b.size());
      })
      // Not in rg's module: device kernel launches so far, per-step device seconds (averaged over
      // `repeats` runs timed with events between steps), and each step's algorithmic cost.
      .def("launches", [](const PyCompiled& self) { return self.c->program->launches(); })
      // Device bytes the program's frames hold now (the compile-time report predates any frame).
      .def("allocated_bytes", [](const PyCompiled& self) { return self.c->program->allocated_bytes(); })
      .def("step_seconds", [](const PyCompiled& self, std::vector<PyTensor> inputs, size_t repeats) {
        auto in = tensors(inputs);
        std::vector<double> secs(self.c->plan.steps.size(), 0.0);
        {
          py::gil_scoped_release nogil;
          auto e = self.c->program->exec();
          for (size_t k = 0; k < in.size(); ++k) e->load(k, in[k]);
          repeats = std::max<size_t>(1, repeats);
          for (size_t r = 0; r < repeats; ++r)
            if (!self.c->program->step_timed(*e, secs)) throw std::runtime_error("this device does not time steps");
        }
        for (auto& s : secs) s /= (double)repeats;
        return secs;
      })
      .def("step_costs", [](const PyCompiled& self) {
        std::vector<std::tuple<std::string, double, double>> out;
        for (auto& c : step_costs(self.c->plan)) out.emplace_back(c.kind, c.flops, c.bytes);
        return out;
      })
      // Not in rg's module: the row chains the CUDA device forms for this plan (none with RGC_ROW_CHAINS=0).
      .def("row_chains", [](const PyCompiled& self) {
        Json a = Json::array();
        for (auto& c : find_row_chains(self.c->plan)) {
          Json j = Json::object();
          auto list = [](const std::vector<size_t>& v) {
            Json x = Json::array();
            for (size_t e : v) x.push(Json((double)e));
            return x;
          };
          j["first"] = Json((double)c.first);
          j["last"] = Json((double)c.last);
          j["members"] = list(c.members);
          j["before"] = list(c.before);
          j["after"] = list(c.after);
          j["rows"] = Json((double)c.rows);
          j["cols"] = Json((double)c.cols);
          Json st = Json::array();
          for (auto& f : c.store) {
            Json x = Json::array();
            for (bool b : f) x.push(Json(b));
            st.push(x);
          }
          j["store"] = st;
          a.push(j);
        }
        return a.dump();
      })
      .def("plan_summary", [](const PyCompiled& self) {
        Json a = Json::array();
        for (auto& st : self.c->plan.steps) {
          Json j = Json::object();
          if (st.fused) {
            std::string ops;
            for (auto& m : st.group.ops) ops += (ops.empty() ? "" : ",") + std::string(m.op.name());
            j["fused"] = ops;
            j["n"] = st.group.n;
            std::vector<size_t> ins, outs;
            for (auto& in : st.group.inputs) ins.push_back(in.slot);
            for (auto& o : st.group.outputs) outs.push_back(o.second);
            j["in"] = Json(ins);
            j["out"] = Json(outs);
          } else {
            j["in"] = Json(st.instr.args);
            j["out"] = Json(std::vector<size_t>{st.instr.dst});
            j["op"] = st.instr.op.name();
            j["shape"] = Json(st.instr.shape);
            Json args = Json::array();
            for (auto& s : st.instr.arg_shapes) args.push(Json(s));
            j["args"] = args;
            j["attr"] = Json(st.instr.op.shape);
            j["flags"] = Json(std::vector<size_t>{(size_t)st.instr.op.flag_a, (size_t)st.instr.op.flag_b});
          }
          a.push(j);
        }
        return a.dump();
      });

  m.def("compile", [](const PyGraph& graph, std::vector<uint32_t> outputs, std::vector<PyTensor> examples, const std::string& level,
                      const std::string& device, const std::string& optimize) {
    OptMode mode;
    if (!parse_opt_mode(optimize, &mode)) throw py::value_error("unknown optimize mode " + optimize);
    std::shared_ptr<Device> dev = module_device(device);
    if (!dev) {
      Json obs = Json::object();
      obs["device"] = device;
      obs["available"] = Json(module_available_devices());
      raise_diag(diag("DEVICE_UNAVAILABLE", "error", Json(), obs, "unknown_device", "verified"));
    }
    Level lv;
    if (!parse_level(level, &lv)) throw py::value_error("unknown validation level " + level);
    for (auto o : outputs)
      if (o >= graph.g.nodes.size()) throw py::index_error("unknown node id " + std::to_string(o));
    auto ex = tensors(examples);
    Graph raw = graph.g;
    return guarded([&] {
      std::unique_ptr<Compiled> c;
      {
        py::gil_scoped_release nogil;
        c = compile_mode(std::move(raw), outputs, ex, lv, dev, mode);
      }
      return PyCompiled{std::move(c)};
    });
  }, py::arg("graph"), py::arg("outputs"), py::arg("examples"), py::arg("level"), py::arg("device"), py::arg("optimize"));

  m.def("available_devices", [] { return module_available_devices(); });
  // Not in rg's module: the optimised graph plans are built from (`gpu` adds the device's own
  // rewrites and memory policy), node by node with the output ids, for tests and plan analysis.
  m.def("_optimized_describe", [](const PyGraph& graph, std::vector<uint32_t> outputs, const std::string& optimize, bool gpu) {
    OptMode mode;
    if (!parse_opt_mode(optimize, &mode)) throw py::value_error("unknown optimize mode " + optimize);
    for (auto id : outputs) graph.check_id(id);
    OptResult r = optimize_mode(graph.g, outputs, mode, gpu);
    auto keep = r.graph.reachable(r.outputs);
    Json nodes = Json::array();
    for (size_t i = 0; i < r.graph.nodes.size(); ++i) {
      const Node& n = r.graph.nodes[i];
      Json j = Json::object();
      j["id"] = i;
      j["op"] = n.op.name();
      j["key"] = n.op.key();
      j["inputs"] = Json(std::vector<size_t>(n.inputs.begin(), n.inputs.end()));
      j["shape"] = Json(n.shape);
      j["live"] = (bool)keep[i];
      nodes.push(j);
    }
    Json out = Json::object();
    out["nodes"] = nodes;
    out["outputs"] = Json(std::vector<size_t>(r.outputs.begin(), r.outputs.end()));
    return out.dump();
  });
  // Not in rg's module: the CPU interpreter validate's device check compares a GPU against
  // (validate.rs:674-705). rg links its own; this module has none and takes one from the
  // embedding process: fn(plan blob bytes, [(bytes, shape, dtype)]) -> [(bytes, shape, dtype)].
  // None removes it (the check then reports itself skipped).
  m.def("_set_reference_runner", [](py::object fn) {
    if (fn.is_none()) {
      set_reference_runner(nullptr);
      return;
    }
    auto holder = std::shared_ptr<py::object>(new py::object(fn), [](py::object* o) {
      if (Py_IsInitialized()) {
        py::gil_scoped_acquire gil;
        delete o;
      }
    });
    set_reference_runner([holder](const Plan& plan, const std::vector<Tensor>& inputs) {
      py::gil_scoped_acquire gil;
      auto blob = encode_plan(plan);
      py::list ins;
      for (auto& t : inputs) ins.append(py::make_tuple(py::bytes((const char*)t.data.data(), t.data.bytes()), t.shape, std::string(dtype_name(t.dtype()))));
      py::object res = (*holder)(py::bytes((const char*)blob.data(), blob.size()), ins);
      std::vector<Tensor> out;
      for (auto item : res) {
        auto tup = item.cast<py::tuple>();
        out.push_back(*make_tensor(tup[0].cast<py::bytes>(), tup[1].cast<std::vector<size_t>>(), tup[2].cast<std::string>()).t);
      }
      return out;
    });
  });
  // Not in rg's module: the equality-saturation search on its own (the unit rg's engine tests
  // exercise), returning (graph, outputs, stats) or None. model: "cpu" | "metal" | "cuda";
  // rule_set: 0 exact, 1 linear, 2 rounding.
  m.def("_egraph_search", [](const PyGraph& graph, std::vector<uint32_t> outputs, const std::string& model, int rule_set, size_t iterations,
                             size_t nodes) -> py::object {
    const CostModel& cm = model == "metal" ? CostModel::METAL : model == "cuda" ? CostModel::CUDA : CostModel::CPU;
    SearchStats st;
    auto found = search(graph.g, outputs, cm, rule_set, iterations, nodes, &st);
    if (!found) return py::none();
    py::dict stats;
    stats["iterations"] = st.iterations;
    stats["egraph_nodes"] = st.egraph_nodes;
    stats["cost_before"] = cm.graph_cost(graph.g, outputs);
    stats["cost_after"] = cm.graph_cost(found->first, found->second);
    PyGraph out{std::move(found->first)};
    return py::make_tuple(py::cast(std::move(out)), found->second, stats);
  });
  module_extra(m);
}
