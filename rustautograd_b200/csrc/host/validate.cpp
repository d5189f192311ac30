// Restates src/validate.rs (line references below are to that file).
#include "validate.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <map>
#include <stdexcept>

#include "plan.h"

namespace rg {

namespace {

constexpr uint64_t VALIDATION_SEED = 0x9E3779B97F4A7C15ull;
constexpr size_t GRAD_CHECK_SAMPLES = 6;
constexpr double GRAD_CHECK_REL_TOL = 1e-4;
constexpr double GRAD_CHECK_ABS_TOL = 1e-7;
constexpr double PERTURBATION = 1e-3;
constexpr double EQUIVALENCE_TOL = 1e-7;
constexpr double DEVICE_TOL = 1e-2;
constexpr size_t MAX_ROOTS = 8;

ReferenceRunner g_reference;

// Shortest decimal form of an f32, read back as f64, so f32 92.7 reports as 92.7
// (tensor.rs `to_json_f64`).
double f32_json(float x) {
  if (!std::isfinite(x)) return (double)x;
  char b[48];
  for (int p = 1; p <= 9; ++p) {
    snprintf(b, sizeof b, "%.*g", p, (double)x);
    if ((float)strtod(b, nullptr) == x) return strtod(b, nullptr);
  }
  return (double)x;
}

double json_value(const Buf& b, size_t i) {
  switch (b.dtype) {
    case DType::F32: return f32_json(b.f32()[i]);
    case DType::F64: return b.f64()[i];
    default: return (double)b.i32()[i];
  }
}

// validate.rs:41-84
struct Stats {
  double min = INFINITY, max = -INFINITY;
  size_t nan = 0, inf = 0, zero = 0, n = 0;
  bool has_fraction = false;
  std::optional<size_t> first_bad;
};

Stats stats(const Buf& b, size_t n) {
  Stats s;
  s.n = n;
  for (size_t i = 0; i < n; ++i) {
    double f = json_value(b, i);
    if (std::isnan(f)) {
      s.nan += 1;
    } else if (std::isinf(f)) {
      s.inf += 1;
    } else {
      s.min = std::min(s.min, f);
      s.max = std::max(s.max, f);
      s.zero += f == 0.0;
      s.has_fraction = s.has_fraction || f != std::trunc(f);
      continue;
    }
    if (!s.first_bad) s.first_bad = i;
  }
  return s;
}

bool any_nonfinite(const Buf& b, size_t n) {
  if (b.dtype == DType::F32) {
    for (size_t i = 0; i < n; ++i)
      if (!std::isfinite(b.f32()[i])) return true;
  } else if (b.dtype == DType::F64) {
    for (size_t i = 0; i < n; ++i)
      if (!std::isfinite(b.f64()[i])) return true;
  }
  return false;
}

// validate.rs:96-130: root-cause rule given finite inputs and a non-finite output.
void classify(const Instr& i, const std::vector<Stats>& args, const Stats& out, std::string* code, std::string* cause, std::string* certainty) {
  *certainty = "verified";
  switch (i.op.kind) {
    case OpKind::Exp: *code = "NUMERIC_OVERFLOW"; *cause = "exponential_overflow"; return;
    case OpKind::Log:
      *code = "DOMAIN_ERROR";
      *cause = args[0].min < 0.0 ? "log_of_negative" : "log_of_zero";
      return;
    case OpKind::Sqrt: *code = "DOMAIN_ERROR"; *cause = "sqrt_of_negative"; return;
    case OpKind::Div:
      if (args[1].zero > 0) { *code = "DIVIDE_BY_ZERO"; *cause = "division_by_zero"; }
      else { *code = "NUMERIC_OVERFLOW"; *cause = "division_overflow"; }
      return;
    case OpKind::Pow: {
      *certainty = args[1].n == 1 ? "verified" : "suspected";
      if (args[0].min < 0.0 && args[1].has_fraction) { *code = "DOMAIN_ERROR"; *cause = "negative_base_fractional_exponent"; }
      else if (args[0].zero > 0 && args[1].min < 0.0) { *code = "DIVIDE_BY_ZERO"; *cause = "zero_base_negative_exponent"; }
      else { *code = "NUMERIC_OVERFLOW"; *cause = "power_overflow"; }
      return;
    }
    case OpKind::Cast: *code = "NUMERIC_OVERFLOW"; *cause = "cast_overflow"; return;
    case OpKind::Add: case OpKind::Sub: case OpKind::Mul: case OpKind::Reduce: case OpKind::MatMul:
      *code = "NUMERIC_OVERFLOW";
      if (out.nan == 0) *cause = "arithmetic_overflow";
      else { *cause = "overflow_then_cancellation"; *certainty = "suspected"; }
      return;
    default: *code = "NONFINITE_OUTPUT"; *cause = "unknown"; *certainty = "unknown";
  }
}

struct Rng {
  uint64_t s;
  uint64_t next() {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
  }
};

Tensor as_f64(const Tensor& t) {
  if (t.dtype() == DType::I32) return t;
  return Tensor::from_f64(DType::F64, t.shape, t.data.to_f64());
}

Json check_status(const std::vector<Json>& d) {
  if (d.empty()) return Json("pass");
  for (auto& x : d)
    if (x.get("severity") && *x.get("severity") == "error") return Json("fail");
  return Json("warn");
}

bool has_error(const std::vector<Json>& d) {
  for (auto& x : d)
    if (x.get("severity") && *x.get("severity") == "error") return true;
  return false;
}

std::vector<Tensor> read_outputs(const Plan& p, Exec& e) {
  std::vector<Tensor> out;
  for (auto& o : p.outputs) out.emplace_back(o.shape, e.prefix(o.slot, o.n));
  return out;
}

}  // namespace

void set_reference_runner(ReferenceRunner r) { g_reference = std::move(r); }

bool parse_level(const std::string& s, Level* l) {
  if (s == "none") *l = Level::None;
  else if (s == "basic") *l = Level::Basic;
  else if (s == "standard") *l = Level::Standard;
  else if (s == "thorough") *l = Level::Thorough;
  else return false;
  return true;
}

Json device_failure(const std::string& device, const std::string& error) {
  Json obs = Json::object();
  obs["device"] = device;
  obs["detail"] = error;
  return diag("DEVICE_EXECUTION_FAILED", "error", Json(), obs, "gpu_reported_a_failure", "verified");
}

// validate.rs:512-513 (`check_inputs`)
void Compiled::check_inputs(const std::vector<Tensor>& inputs) const {
  std::vector<uint32_t> ids;
  for (size_t i = 0; i < raw.nodes.size(); ++i)
    if (raw.nodes[i].op.kind == OpKind::Input) ids.push_back((uint32_t)i);
  if (ids.size() != inputs.size()) {
    Json obs = Json::object();
    obs["expected_inputs"] = ids.size();
    obs["actual_inputs"] = inputs.size();
    obs["recompile_required"] = true;
    throw DiagError(diag("INPUT_SIGNATURE_MISMATCH", "error", Json(), obs, "input_count_changed", "verified"));
  }
  for (size_t k = 0; k < ids.size(); ++k) {
    const Node& n = raw.nodes[ids[k]];
    const Tensor& t = inputs[k];
    if (n.shape != t.shape || n.dtype != t.dtype()) {
      Json obs = Json::object();
      obs["input_index"] = k;
      obs["expected_shape"] = Json(n.shape);
      obs["actual_shape"] = Json(t.shape);
      obs["expected_dtype"] = dtype_name(n.dtype);
      obs["actual_dtype"] = dtype_name(t.dtype());
      obs["recompile_required"] = true;
      throw DiagError(diag("INPUT_SIGNATURE_MISMATCH", "error", raw.node_json(ids[k]), obs, "input_signature_changed", "verified"));
    }
  }
}

// validate.rs:515-535
std::vector<Tensor> Compiled::try_call(const std::vector<Tensor>& inputs) const {
  std::unique_ptr<Exec> e;
  try {
    e = program->exec();
  } catch (const std::exception& ex) {
    throw DiagError(device_failure(device->name(), ex.what()));
  }
  for (size_t k = 0; k < inputs.size(); ++k) e->load(k, inputs[k]);
  e->step();
  if (auto f = e->failure()) throw DiagError(device_failure(device->name(), *f));
  return read_outputs(plan, *e);
}

std::vector<uint32_t> Compiled::raw_outputs() const {
  std::vector<uint32_t> all = outputs;
  for (auto& r : raw.grads) all.push_back(r.grad);
  return all;
}

// validate.rs:541-565 with the NonFinite observer of 132-230, one plan step at a time.
Compiled::Observed Compiled::observed(const std::vector<Tensor>& inputs) const {
  Observed o;
  auto keep = raw.reachable(raw_outputs());
  for (size_t id = 0; id < raw.nodes.size(); ++id) {
    const Node& n = raw.nodes[id];
    const Tensor* t = nullptr;
    if (n.op.kind == OpKind::Input) t = &inputs[n.op.index];
    else if (n.op.kind == OpKind::Const) t = n.op.value.get();
    else continue;
    if (keep[id] && !t->is_finite()) {
      Stats s = stats(t->data, t->n());
      Json obs = Json::object();
      obs["dtype"] = dtype_name(n.dtype);
      obs["shape"] = Json(n.shape);
      obs["contains_inf"] = s.inf > 0;
      obs["contains_nan"] = s.nan > 0;
      obs["nonfinite_count"] = s.nan + s.inf;
      obs["first_bad_index"] = s.first_bad ? Json(*s.first_bad) : Json();
      o.roots.push_back(diag("NONFINITE_INPUT", "error", raw.node_json((uint32_t)id), obs, "nonfinite_value_supplied", "verified"));
    }
  }
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (!raw_program_) raw_program_ = device->compile(raw_plan);
  }
  auto e = raw_program_->exec();
  for (size_t k = 0; k < inputs.size(); ++k) e->load(k, inputs[k]);
  for (size_t k = 0; k < raw_plan.steps.size(); ++k) {
    e->step_at(k);
    const Step& st = raw_plan.steps[k];
    if (st.fused) continue;  // reference plans have no groups
    const Instr& i = st.instr;
    // Index check (validate.rs:177-190).
    size_t dim = 0;
    if (i.op.kind == OpKind::Take) dim = i.arg_shapes[0][i.op.index];
    else if (i.op.kind == OpKind::TakeAlong) dim = i.arg_shapes[0].back();
    if (dim) {
      size_t n = product(i.arg_shapes[1]);
      Stats s = stats(e->prefix(i.args[1], n), n);
      if (n > 0 && (s.min < 0.0 || s.max >= (double)dim) && o.hard.size() < MAX_ROOTS) {
        Json obs = Json::object();
        obs["index_min"] = s.min;
        obs["index_max"] = s.max;
        obs["axis_size"] = dim;
        obs["behavior_at_runtime"] = "clamped";
        o.hard.push_back(diag("INDEX_OUT_OF_RANGE", "error", raw.node_json(i.node), obs, "index_outside_axis", "verified"));
      }
    }
    if (i.op.is_control_flow()) {
      // Bodies run as one step here; a non-finite value they produce is reported at the
      // control-flow node itself.
      for (auto& [index, slot] : i.outs) {
        (void)index;
        size_t n = product(raw_plan.slots[slot].second == 0 ? std::vector<size_t>{0} : std::vector<size_t>{raw_plan.slots[slot].second});
        if (any_nonfinite(e->prefix(slot, n), n) && o.roots.size() < MAX_ROOTS) {
          Json obs = Json::object();
          obs["dtype"] = dtype_name(raw_plan.slots[slot].first);
          o.roots.push_back(diag("NONFINITE_OUTPUT", "error", raw.node_json(i.node), obs, "unknown", "unknown"));
          break;
        }
      }
      continue;
    }
    Buf out = e->prefix(i.dst, i.n);
    if (!any_nonfinite(out, i.n)) continue;
    std::vector<size_t> ns;
    std::vector<Buf> argv;
    std::vector<Stats> args;
    for (size_t a = 0; a < i.args.size(); ++a) {
      ns.push_back(product(i.arg_shapes[a]));
      argv.push_back(e->prefix(i.args[a], ns.back()));
      args.push_back(stats(argv.back(), ns.back()));
    }
    bool propagated = false;
    for (auto& a : args) propagated = propagated || a.first_bad.has_value();
    if (propagated) {
      o.propagated += 1;
      continue;
    }
    if (o.roots.size() == MAX_ROOTS) continue;
    Stats os = stats(out, i.n);
    std::string code, cause, certainty;
    classify(i, args, os, &code, &cause, &certainty);
    size_t bad = *os.first_bad;
    bool elementwise = i.op.is_unary_elementwise() || i.op.is_binary_elementwise();
    Json witness;
    if (elementwise && i.mode != Mode::General) {
      witness = Json::object();
      Json vals = Json::array();
      for (size_t a = 0; a < argv.size(); ++a) vals.push(jnum(json_value(argv[a], ns[a] == i.n ? bad : 0)));
      witness["index"] = bad;
      witness["inputs"] = vals;
      witness["output"] = jnum(json_value(out, bad));
    }
    Json obs = Json::object();
    obs["dtype"] = dtype_name(i.dtype);
    Json ins = Json::array();
    for (size_t a = 0; a < args.size(); ++a) {
      Json x = Json::object();
      x["shape"] = Json(i.arg_shapes[a]);
      x["min"] = jnum(args[a].min);
      x["max"] = jnum(args[a].max);
      x["contains_zero"] = args[a].zero > 0;
      ins.push(x);
    }
    obs["inputs"] = ins;
    obs["output_shape"] = Json(i.shape);
    obs["output_contains_inf"] = os.inf > 0;
    obs["output_contains_nan"] = os.nan > 0;
    obs["nonfinite_count"] = os.nan + os.inf;
    obs["witness"] = witness;
    if (args.size() == 1) {
      obs["input_max"] = jnum(args[0].max);
      obs["input_min"] = jnum(args[0].min);
      if (i.op.kind == OpKind::Exp) obs["overflow_threshold"] = jnum(i.dtype == DType::F32 ? 88.722839 : 709.782712);
    }
    o.roots.push_back(diag(code, "error", raw.node_json(i.node), obs, cause, certainty));
  }
  if (auto f = e->failure()) throw DiagError(device_failure(device->name(), *f));
  o.values = read_outputs(raw_plan, *e);
  return o;
}

// validate.rs:573-600
std::pair<Json, std::vector<Json>> Compiled::gradient_stats(const std::vector<Tensor>& vals) const {
  Json out = Json::array();
  std::vector<Json> diags;
  for (size_t k = 0; k < raw.grads.size(); ++k) {
    const GradRecord& r = raw.grads[k];
    auto v = vals[outputs.size() + k].data.to_f64();
    if (v.empty()) continue;
    size_t zeros = 0;
    double sq = 0, max_abs = 0;
    for (double x : v) {
      zeros += x == 0.0;
      sq += x * x;
      if (std::fabs(x) > max_abs || std::isnan(x)) max_abs = std::fabs(x);
    }
    Json g = Json::object();
    g["output_node"] = r.y;
    g["wrt_node"] = r.wrt;
    g["grad_node"] = r.grad;
    g["source"] = raw.nodes[r.wrt].source ? Json(*raw.nodes[r.wrt].source) : Json();
    g["norm"] = jnum(std::sqrt(sq));
    g["rms"] = jnum(std::sqrt(sq / (double)std::max<size_t>(v.size(), 1)));
    g["max_abs"] = jnum(max_abs);
    g["zero_ratio"] = jnum((double)zeros / (double)v.size());
    out.push(g);
    bool is_const = raw.nodes[r.grad].op.kind == OpKind::Const;
    if (zeros == v.size() && !is_const) {
      Json obs = Json::object();
      obs["wrt_node"] = r.wrt;
      obs["zero_ratio"] = 1.0;
      obs["elements"] = v.size();
      diags.push_back(diag("GRAD_ALL_ZERO", "warning", raw.node_json(r.grad), obs, "zero_gradient_at_sample", "suspected"));
    }
  }
  return {out, diags};
}

// validate.rs:604-632
std::optional<std::vector<Tensor>> Compiled::scanned(const std::vector<Tensor>& inputs) const {
  if (!device->fuse().gpu) return std::nullopt;
  for (auto& t : inputs)
    if (!t.is_finite()) return std::nullopt;
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (!scan_program_) {
      std::vector<uint32_t> all = raw_outputs();
      OptResult opt = optimize_mode(raw, all, mode, true);
      scan_plan_ = Plan::build_fused(opt.graph, opt.outputs, device->fuse());
      scan_program_ = device->compile(scan_plan_);
    }
  }
  auto e = scan_program_->exec();
  for (size_t k = 0; k < inputs.size(); ++k) e->load(k, inputs[k]);
  std::vector<int32_t> flags(2 * scan_plan_.steps.size(), 0);
  if (!scan_program_->step_checked(*e, flags)) return std::nullopt;
  if (auto f = e->failure()) throw DiagError(device_failure(device->name(), *f));
  for (int32_t f : flags)
    if (f) return std::nullopt;
  return read_outputs(scan_plan_, *e);
}

Json Compiled::check(const std::vector<Tensor>& inputs) const {
  Observed o;
  bool on_device = false;
  if (auto values = scanned(inputs)) {
    // Nothing non-finite and every index in range: no roots to look for.
    o.values = std::move(*values);
    on_device = true;
  } else {
    o = observed(inputs);
  }
  std::vector<size_t> bad_outputs;
  for (size_t k = 0; k < outputs.size(); ++k)
    if (!o.values[k].is_finite()) bad_outputs.push_back(k);
  if (bad_outputs.empty()) {
    for (auto& r : o.roots) {
      r["severity"] = "warning";
      r["status"] = "warning";
      r["masked"] = true;
    }
  }
  auto gs = gradient_stats(o.values);
  std::string status = (!bad_outputs.empty() || !o.hard.empty()) ? "validation_failed"
                       : (!o.roots.empty() || !gs.second.empty()) ? "warning" : "ok";
  size_t found = o.roots.size();
  Json d = Json::array();
  for (auto& r : o.roots) d.push(r);
  for (auto& r : gs.second) d.push(r);
  for (auto& r : o.hard) d.push(r);
  Json out = Json::object();
  out["status"] = status;
  Json nf = Json::object();
  nf["root_nodes"] = found;
  nf["propagated_nodes"] = o.propagated;
  nf["affected_outputs"] = Json(bad_outputs);
  nf["scan"] = on_device ? "device" : "stepwise";
  out["nonfinite"] = nf;
  out["gradients"] = gs.first;
  out["diagnostics"] = d;
  return out;
}

// validate.rs:637-670: optimised plan against the plain graph, both in f64.
Json Compiled::optimizer_check(const std::vector<Tensor>& examples) const {
  Graph shadow = raw.to_f64();
  std::vector<Tensor> inputs;
  for (auto& t : examples) inputs.push_back(as_f64(t));
  std::vector<const Tensor*> ptrs;
  for (auto& t : inputs) ptrs.push_back(&t);
  OptResult opt = optimize_mode(shadow, outputs, mode, device->fuse().gpu);
  auto fast = run_once(*device, Plan::build_fused(opt.graph, opt.outputs, device->fuse()), ptrs);
  auto reference = run_once(*device, Plan::build(shadow, outputs, false), ptrs);
  double max_rel = 0;
  for (size_t k = 0; k < fast.size(); ++k) {
    auto va = fast[k].data.to_f64(), vb = reference[k].data.to_f64();
    double scale = 1e-30;
    for (double v : vb)
      if (std::isfinite(v)) scale = std::max(scale, std::fabs(v));
    for (size_t j = 0; j < va.size(); ++j) {
      double x = va[j], y = vb[j];
      if (x == y || (std::isnan(x) && std::isnan(y))) continue;
      double rel = std::fabs(x - y) / scale;
      max_rel = std::isnan(rel) ? INFINITY : std::max(max_rel, rel);
      if (!(rel <= EQUIVALENCE_TOL)) {
        Json obs = Json::object();
        obs["output_index"] = k;
        obs["element"] = j;
        obs["optimized"] = jnum(x);
        obs["reference"] = jnum(y);
        obs["relative_error"] = jnum(rel);
        obs["tolerance"] = EQUIVALENCE_TOL;
        obs["precision"] = "float64";
        throw DiagError(diag("OPTIMIZER_MISMATCH", "error", raw.node_json(outputs[k]), obs, "optimized_plan_disagrees_with_reference", "verified"));
      }
    }
  }
  Json info = Json::object();
  info["max_relative_error"] = jnum(max_rel);
  info["tolerance"] = EQUIVALENCE_TOL;
  info["precision"] = "float64";
  return info;
}

// validate.rs:674-705, against rg's CPU interpreter when the process provides one.
std::pair<Json, std::vector<Json>> Compiled::device_check(const std::vector<Tensor>& examples) const {
  std::vector<Json> diags;
  if (!g_reference) {
    Json s = Json::object();
    s["skipped"] = "no_cpu_reference_in_this_process";
    return {s, diags};
  }
  OptResult opt = optimize_mode(raw, outputs, mode, device->fuse().gpu);
  Plan cpu_plan = Plan::build_fused(opt.graph, opt.outputs, Fuse::DEFAULT());
  std::vector<Tensor> cpu = g_reference(cpu_plan, examples);
  std::vector<Tensor> gpu;
  try {
    gpu = try_call(examples);
  } catch (const DiagError& d) {
    Json s = Json::object();
    s["skipped"] = "device_failed";
    diags.push_back(d.diag);
    return {s, diags};
  }
  double max_rel = 0;
  for (size_t k = 0; k < gpu.size(); ++k) {
    auto vg = gpu[k].data.to_f64(), vc = cpu[k].data.to_f64();
    double scale = 1e-30;
    for (double v : vc)
      if (std::isfinite(v)) scale = std::max(scale, std::fabs(v));
    for (size_t j = 0; j < vg.size(); ++j) {
      double x = vg[j], y = vc[j];
      if (x == y || (std::isnan(x) && std::isnan(y))) continue;
      double rel = std::fabs(x - y) / scale;
      if (std::isnan(rel)) rel = INFINITY;
      max_rel = std::max(max_rel, rel);
      if (rel > DEVICE_TOL && diags.empty()) {
        Json obs = Json::object();
        obs["output_index"] = k;
        obs["element"] = j;
        obs[device->name()] = jnum(x);
        obs["cpu"] = jnum(y);
        obs["relative_error"] = jnum(rel);
        obs["tolerance"] = DEVICE_TOL;
        diags.push_back(diag("DEVICE_MISMATCH", "warning", raw.node_json(outputs[k]), obs, device->name() + "_result_differs_from_cpu", "suspected"));
      }
    }
  }
  Json info = Json::object();
  info["max_relative_error"] = jnum(max_rel);
  info["tolerance"] = DEVICE_TOL;
  return {info, diags};
}

// validate.rs:708-772: central differences in f64 against every recorded gradient.
std::pair<Json, std::vector<Json>> Compiled::grad_check(const std::vector<Tensor>& examples) const {
  Graph shadow = raw.to_f64();
  std::vector<Tensor> inputs64;
  for (auto& t : examples) inputs64.push_back(as_f64(t));
  Rng rng{VALIDATION_SEED};
  size_t checked = 0;
  Json skipped = Json::array();
  double max_rel = 0;
  std::vector<Json> diags;
  for (auto& r : raw.grads) {
    auto keep = raw.reachable({r.y});
    const Node& w = raw.nodes[r.wrt];
    if (w.op.kind != OpKind::Input) {
      Json s = Json::object();
      s["wrt_node"] = r.wrt;
      s["reason"] = "wrt_is_not_an_input";
      skipped.push(s);
      continue;
    }
    size_t k = w.op.index;
    if (raw.nodes[r.grad].op.kind == OpKind::Const) {
      Json s = Json::object();
      s["wrt_node"] = r.wrt;
      s["reason"] = "disconnected";
      skipped.push(s);
      continue;
    }
    bool soft = false;
    for (size_t i = 0; i < raw.nodes.size(); ++i)
      if (keep[i] && (raw.nodes[i].op.is_nonsmooth() || raw.nodes[i].op.kind == OpKind::StopGradient)) soft = true;
    std::string certainty = soft ? "suspected" : "verified";
    Plan analytic_plan = Plan::build(shadow, {r.grad}, true);
    Plan y_plan = Plan::build(shadow, {r.y}, true);
    std::vector<const Tensor*> ptrs;
    for (auto& t : inputs64) ptrs.push_back(&t);
    auto analytic = run_once(*device, analytic_plan, ptrs)[0].data.to_f64();
    auto prog = device->compile(y_plan);
    auto ye = prog->exec();
    for (size_t j = 0; j < inputs64.size(); ++j) ye->load(j, inputs64[j]);
    Tensor probe = inputs64[k];
    auto base = inputs64[k].data.to_f64();
    for (size_t s = 0; s < std::min(GRAD_CHECK_SAMPLES, base.size()); ++s) {
      size_t e = base.size() <= GRAD_CHECK_SAMPLES ? s : (size_t)(rng.next() % base.size());
      double h = 1e-6 * std::max(std::fabs(base[e]), 1.0);
      auto eval_at = [&](double x) {
        probe.data.f64()[e] = x;
        ye->load(k, probe);
        ye->step();
        return ye->scalar(y_plan.outputs[0].slot);
      };
      double up = eval_at(base[e] + h), down = eval_at(base[e] - h);
      probe.data.f64()[e] = base[e];
      double numeric = (up - down) / (2.0 * h);
      if (!std::isfinite(numeric) || !std::isfinite(analytic[e])) continue;
      checked += 1;
      double err = std::fabs(numeric - analytic[e]);
      double rel = err / std::max(std::max(std::fabs(numeric), std::fabs(analytic[e])), 1e-12);
      max_rel = std::max(max_rel, err <= GRAD_CHECK_ABS_TOL ? 0.0 : rel);
      if (err > GRAD_CHECK_ABS_TOL && rel > GRAD_CHECK_REL_TOL) {
        Json obs = Json::object();
        obs["wrt_node"] = r.wrt;
        obs["element"] = e;
        obs["analytic"] = jnum(analytic[e]);
        obs["numeric"] = jnum(numeric);
        obs["relative_error"] = jnum(rel);
        obs["tolerance"] = GRAD_CHECK_REL_TOL;
        obs["finite_difference_h"] = h;
        obs["seed"] = (unsigned long long)VALIDATION_SEED;
        std::string severity = certainty == "verified" ? "error" : "warning";
        diags.push_back(diag("GRADIENT_MISMATCH", severity, raw.node_json(r.grad), obs, "analytic_gradient_disagrees_with_finite_difference", certainty));
        break;
      }
    }
  }
  Json info = Json::object();
  info["elements_checked"] = checked;
  info["max_relative_error"] = jnum(max_rel);
  info["skipped"] = skipped;
  return {info, diags};
}

// validate.rs:774-797
std::pair<Json, std::vector<Json>> Compiled::perturbation_check(const std::vector<Tensor>& examples) const {
  Rng rng{VALIDATION_SEED ^ 0xABCD};
  std::vector<Tensor> moved;
  for (auto& t : examples) {
    if (t.dtype() == DType::I32) {
      moved.push_back(t);  // tokens and keys are identities, not magnitudes
      continue;
    }
    auto v = t.data.to_f64();
    for (auto& x : v) x = x * (1.0 + (rng.next() % 2 == 0 ? PERTURBATION : -PERTURBATION));
    moved.push_back(Tensor::from_f64(t.dtype(), t.shape, v));
  }
  Observed o = observed(moved);
  std::vector<Json> diags;
  for (auto d : o.roots) {
    d["severity"] = "warning";
    d["status"] = "warning";
    Json trig = Json::object();
    trig["kind"] = "input_perturbation";
    trig["relative_magnitude"] = PERTURBATION;
    trig["seed"] = (unsigned long long)VALIDATION_SEED;
    d["trigger"] = trig;
    diags.push_back(d);
  }
  Json info = Json::object();
  info["relative_magnitude"] = PERTURBATION;
  return {info, diags};
}

// validate.rs:799-873
Json Compiled::validate(const std::vector<Tensor>& examples) {
  Json checks = Json::array();
  {
    Json c = Json::object();
    c["name"] = "static";
    c["status"] = "pass";
    c["detail"] = "shape and dtype inference passed during tracing";
    checks.push(c);
  }
  std::vector<Json> diagnostics = raw.notes;
  Json gradients = Json::array();
  if (level >= Level::Basic) {
    try {
      auto out = try_call(examples);
      Json shapes = Json::array();
      for (auto& t : out) shapes.push(Json(t.shape));
      Json c = Json::object();
      c["name"] = "test_run";
      c["status"] = "pass";
      c["output_shapes"] = shapes;
      checks.push(c);
    } catch (const DiagError& d) {
      Json c = Json::object();
      c["name"] = "test_run";
      c["status"] = "fail";
      checks.push(c);
      diagnostics.push_back(d.diag);
    }
  }
  if (level >= Level::Standard) {
    Json found = check(examples);
    std::vector<Json> ds = found.get("diagnostics")->items();
    Json c = Json::object();
    c["name"] = "finite";
    c["status"] = check_status(ds);
    c["nonfinite"] = *found.get("nonfinite");
    checks.push(c);
    gradients = *found.get("gradients");
    diagnostics.insert(diagnostics.end(), ds.begin(), ds.end());
    try {
      Json info = optimizer_check(examples);
      Json oc = Json::object();
      oc["name"] = "optimizer_equivalence";
      oc["status"] = "pass";
      oc["detail"] = info;
      checks.push(oc);
    } catch (const DiagError& d) {
      Json oc = Json::object();
      oc["name"] = "optimizer_equivalence";
      oc["status"] = "fail";
      checks.push(oc);
      diagnostics.push_back(d.diag);
    }
    if (device->name() != "cpu") {
      auto [info, dd] = device_check(examples);
      Json dc = Json::object();
      dc["name"] = "device_equivalence";
      dc["status"] = check_status(dd);
      dc["detail"] = info;
      checks.push(dc);
      diagnostics.insert(diagnostics.end(), dd.begin(), dd.end());
    }
  }
  if (level >= Level::Thorough) {
    auto [info, ds] = grad_check(examples);
    Json c = Json::object();
    c["name"] = "grad_check";
    c["status"] = check_status(ds);
    c["detail"] = info;
    checks.push(c);
    diagnostics.insert(diagnostics.end(), ds.begin(), ds.end());
    auto [pinfo, pds] = perturbation_check(examples);
    Json p = Json::object();
    p["name"] = "input_perturbation";
    p["status"] = check_status(pds);
    p["detail"] = pinfo;
    checks.push(p);
    diagnostics.insert(diagnostics.end(), pds.begin(), pds.end());
  }
  std::string status = has_error(diagnostics) ? "validation_failed" : diagnostics.empty() ? "ok" : "warning";
  Json rep = Json::object();
  rep["status"] = status;
  rep["device"] = device->name();
  Json graph = Json::object();
  graph["optimization"] = opt_stats.json();
  graph["steps"] = plan.steps.size();
  graph["fused_groups"] = plan.n_fused();
  graph["fused_ops"] = plan.n_fused_ops();
  rep["graph"] = graph;
  Json mem = Json::object();
  mem["intermediate_bytes_without_reuse"] = plan.naive_bytes;
  mem["intermediate_bytes_planned"] = plan.planned_bytes();
  mem["peak_live_bytes"] = plan.peak_live_bytes;
  if (program) mem["device_bytes_allocated"] = program->allocated_bytes();
  rep["memory"] = mem;
  rep["checks"] = checks;
  rep["gradients"] = gradients;
  Json dj = Json::array();
  for (auto& d : diagnostics) dj.push(d);
  rep["diagnostics"] = dj;
  Json repro = Json::object();
  static const char* names[] = {"none", "basic", "standard", "thorough"};
  repro["level"] = names[(int)level];
  repro["seed"] = (unsigned long long)VALIDATION_SEED;
  rep["repro"] = repro;
  return rep;
}

// validate.rs:876-919
Json Compiled::profile(const std::vector<Tensor>& inputs, size_t repeats) const {
  repeats = std::max<size_t>(repeats, 1);
  std::vector<double> seconds(plan.steps.size(), 0.0);
  auto e = program->exec();
  for (size_t k = 0; k < inputs.size(); ++k) e->load(k, inputs[k]);
  Json breakdown = program->breakdown(*e, repeats);
  for (size_t r = 0; r < repeats; ++r) {
    if (!program->step_timed(*e, seconds)) {
      auto t0 = std::chrono::steady_clock::now();
      for (size_t k = 0; k < plan.steps.size(); ++k) {
        auto s0 = std::chrono::steady_clock::now();
        e->step_at(k);
        seconds[k] += std::chrono::duration<double>(std::chrono::steady_clock::now() - s0).count();
      }
      (void)t0;
    }
  }
  std::map<std::string, std::tuple<double, size_t>> rows;
  for (size_t k = 0; k < plan.steps.size(); ++k) {
    const Step& s = plan.steps[k];
    std::string key;
    if (s.fused) {
      key = "fused[";
      for (size_t m = 0; m < s.group.ops.size(); ++m) key += (m ? "," : "") + std::string(s.group.ops[m].op.name());
      key += "] n=" + std::to_string(s.group.n);
    } else {
      key = std::string(s.instr.op.name()) + " " + Json(s.instr.shape).dump() + " <- [";
      for (size_t a = 0; a < s.instr.arg_shapes.size(); ++a) key += (a ? ", " : "") + Json(s.instr.arg_shapes[a]).dump();
      key += "]";
    }
    auto& row = rows[key];
    std::get<0>(row) += seconds[k];
    std::get<1>(row) += 1;
  }
  double total = 0;
  for (double t : seconds) total += t;
  std::vector<std::pair<std::string, std::tuple<double, size_t>>> list(rows.begin(), rows.end());
  std::stable_sort(list.begin(), list.end(), [](auto& a, auto& b) { return std::get<0>(a.second) > std::get<0>(b.second); });
  Json top = Json::array();
  for (auto& [k, v] : list) {
    Json r = Json::object();
    r["operation"] = k;
    r["count"] = std::get<1>(v);
    r["microseconds_per_run"] = std::get<0>(v) / (double)repeats * 1e6;
    r["share"] = total > 0 ? std::get<0>(v) / total : 0.0;
    top.push(r);
  }
  Json out = Json::object();
  out["repeats"] = repeats;
  out["microseconds_per_run"] = total / (double)repeats * 1e6;
  out["operations"] = top;
  out["breakdown"] = breakdown;
  return out;
}

void Compiled::validate_spec(const RunSpec& spec) const {
  for (auto& [i, o] : spec.state) {
    uint32_t input = 0;
    for (size_t n = 0; n < raw.nodes.size(); ++n)
      if (raw.nodes[n].op.kind == OpKind::Input && raw.nodes[n].op.index == i) input = (uint32_t)n;
    uint32_t out = outputs[o];
    if (raw.shape(input) != raw.shape(out) || raw.dtype(input) != raw.dtype(out)) {
      Json obs = Json::object();
      obs["input_index"] = i;
      obs["output_index"] = o;
      obs["input_shape"] = Json(raw.shape(input));
      obs["output_shape"] = Json(raw.shape(out));
      obs["input_dtype"] = dtype_name(raw.dtype(input));
      obs["output_dtype"] = dtype_name(raw.dtype(out));
      throw DiagError(diag("STATE_CONTRACT_VIOLATION", "error", raw.node_json(out), obs, "returned_state_differs_from_input_state", "verified"));
    }
  }
}

// validate.rs:937-951
RunOut Compiled::run_refs(const RunSpec& spec, const std::vector<const Tensor*>& state, const std::vector<std::vector<const Tensor*>>& batches,
                          size_t steps) const {
  auto owned = [](const std::vector<const Tensor*>& v) {
    std::vector<Tensor> out;
    out.reserve(v.size());
    for (const Tensor* t : v) out.push_back(*t);
    return out;
  };
  std::unique_ptr<Exec> e;
  try {
    e = program->exec();
  } catch (const std::exception& ex) {
    RunOut r;
    r.state = owned(state);
    r.history.assign(spec.history.size(), {});
    r.device_error = ex.what();
    return r;
  }
  RunOut r;
  if (e->run(spec, state, batches, steps, &r)) return r;
  std::vector<std::vector<Tensor>> bs;
  for (auto& b : batches) bs.push_back(owned(b));
  return run_loop(plan, *e, spec, owned(state), bs, steps);
}

RunOut Compiled::run(const RunSpec& spec, const std::vector<Tensor>& state, const std::vector<std::vector<Tensor>>& batches, size_t steps) const {
  std::vector<const Tensor*> sp;
  for (auto& t : state) sp.push_back(&t);
  std::vector<std::vector<const Tensor*>> bp;
  for (auto& b : batches) {
    bp.emplace_back();
    for (auto& t : b) bp.back().push_back(&t);
  }
  RunOut r = run_refs(spec, sp, bp, steps);
  if (r.state_outputs_elided) {
    for (size_t k = 0; k < spec.state.size() && k < r.state.size(); ++k)
      if (spec.state[k].second < r.outputs.size()) r.outputs[spec.state[k].second] = r.state[k];
    r.state_outputs_elided = false;
  }
  return r;
}

// validate.rs:955-970
bool Compiled::replay(const RunSpec& spec, const std::vector<Tensor>& state, const std::vector<std::vector<Tensor>>& batches, size_t steps,
                      size_t* step, size_t* batch, std::vector<Tensor>* before) const {
  std::vector<Tensor> cur = state;
  for (size_t k = 0; k < steps; ++k) {
    size_t b = batches.empty() ? 0 : k % batches.size();
    std::vector<std::vector<Tensor>> slice;
    if (!batches.empty()) slice.push_back(batches[b]);
    RunOut out = run(spec, cur, slice, 1);
    if (out.device_error) return false;
    bool bad = false;
    for (auto& t : out.state) bad = bad || !t.is_finite();
    for (auto& t : out.outputs) bad = bad || !t.is_finite();
    if (bad) {
      *step = k;
      *batch = b;
      *before = cur;
      return true;
    }
    cur = out.state;
  }
  return false;
}

namespace {

std::unique_ptr<Compiled> build(const Graph& raw, const std::vector<uint32_t>& outputs, const std::vector<Tensor>& examples, Level level,
                                std::shared_ptr<Device> device, OptMode mode) {
  auto c = std::make_unique<Compiled>();
  OptResult opt = optimize_mode(raw, outputs, mode, device->fuse().gpu);
  c->plan = Plan::build_fused(opt.graph, opt.outputs, device->fuse());
  try {
    c->program = device->compile(c->plan);
  } catch (const std::exception& ex) {
    Json obs = Json::object();
    obs["device"] = device->name();
    obs["detail"] = ex.what();
    throw DiagError(diag("DEVICE_UNAVAILABLE", "error", Json(), obs, device->name() + "_device_memory_or_kernel_compilation_failed", "verified"));
  }
  std::vector<uint32_t> all = outputs;
  for (auto& r : raw.grads) all.push_back(r.grad);
  c->raw_plan = Plan::build(raw, all, false);
  c->raw = raw;
  c->outputs = outputs;
  c->level = level;
  c->device = device;
  c->mode = mode;
  c->opt_stats = opt.stats;
  c->check_inputs(examples);
  c->report = c->validate(examples);
  return c;
}

bool has_equivalence_failure(const Json& report) {
  const Json* d = report.get("diagnostics");
  if (!d) return false;
  for (auto& x : d->items())
    if (x.get("code") && *x.get("code") == "OPTIMIZER_MISMATCH") return true;
  return false;
}

void push_diagnostic(Json& report, Json d) {
  report["diagnostics"].push(std::move(d));
  if (report["status"] == "ok") report["status"] = "warning";
}

}  // namespace

// validate.rs:393-473
std::unique_ptr<Compiled> compile_mode(Graph raw, std::vector<uint32_t> outputs, const std::vector<Tensor>& examples, Level level,
                                       std::shared_ptr<Device> device, OptMode mode) {
  if (mode == OptMode::Auto) {
    auto standard = build(raw, outputs, examples, Level::None, device, OptMode::Standard);
    auto searched = compile_mode(raw, outputs, examples, Level::Basic, device, OptMode::SearchLinear);
    bool rewritten = searched->opt_stats.search && searched->opt_stats.search->accepted;
    bool use_search = false;
    Json timing;
    if (rewritten) {
      try { standard->try_call(examples); searched->try_call(examples); } catch (...) {}
      std::vector<double> ta, tb;
      auto started = std::chrono::steady_clock::now();
      for (int round = 0; round < 7; ++round) {
        for (int k : {round % 2, 1 - round % 2}) {
          auto t0 = std::chrono::steady_clock::now();
          try { (k == 0 ? standard : searched)->try_call(examples); } catch (...) {}
          (k == 0 ? ta : tb).push_back(std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
        }
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - started).count() > 0.5) break;
      }
      std::sort(ta.begin(), ta.end());
      std::sort(tb.begin(), tb.end());
      double a = ta[ta.size() / 2], b = tb[tb.size() / 2];
      use_search = a / b >= 1.05;
      timing = Json::object();
      timing["standard_seconds"] = a;
      timing["rewritten_seconds"] = b;
    }
    standard.reset();
    searched.reset();
    auto c = compile_mode(raw, outputs, examples, level, device, use_search ? OptMode::SearchLinear : OptMode::Standard);
    Json a = Json::object();
    a["chosen"] = use_search ? "search-linear" : "standard";
    a["rewrite_proposed"] = rewritten;
    a["timing"] = timing;
    c->report["auto"] = a;
    return c;
  }
  auto c = build(raw, outputs, examples, level, device, mode);
  bool rewritten = c->opt_stats.search && c->opt_stats.search->accepted;
  if (rewritten && has_equivalence_failure(c->report)) {
    Json rejected;
    for (auto& x : c->report["diagnostics"].items())
      if (x.get("code") && *x.get("code") == "OPTIMIZER_MISMATCH") rejected = x;
    c = build(raw, outputs, examples, level, device, OptMode::Standard);
    if (!rejected.is_null()) {
      push_diagnostic(c->report, diag("REWRITE_REJECTED", "warning", *rejected.get("node"), *rejected.get("observation"),
                                      "rewritten_program_failed_the_equivalence_check_standard_plan_used", "verified"));
    }
  }
  return c;
}

}  // namespace rg
