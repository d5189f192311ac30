// IR construction and inference; restates src/graph.rs (line references below are to that file).
#include "graph.h"

#include <algorithm>
#include <cstdio>
#include <set>

#include "optimize.h"
#include "plan.h"

namespace rg {

// graph.rs:117-172
const char* Op::name() const {
  switch (kind) {
    case OpKind::Input: return "input";
    case OpKind::Const: return "const";
    case OpKind::Neg: return "neg";
    case OpKind::Exp: return "exp";
    case OpKind::Log: return "log";
    case OpKind::Sqrt: return "sqrt";
    case OpKind::Sin: return "sin";
    case OpKind::Cos: return "cos";
    case OpKind::Tanh: return "tanh";
    case OpKind::Abs: return "abs";
    case OpKind::Sign: return "sign";
    case OpKind::Add: return "add";
    case OpKind::Sub: return "sub";
    case OpKind::Mul: return "mul";
    case OpKind::Div: return "div";
    case OpKind::Pow: return "pow";
    case OpKind::Max: return "maximum";
    case OpKind::Min: return "minimum";
    case OpKind::Gt: return "gt";
    case OpKind::Ge: return "ge";
    case OpKind::Where: return "where";
    case OpKind::MatMul: return "matmul";
    case OpKind::MatMulT: return "matmul_t";
    case OpKind::Reduce:
      return reduce == ReduceKind::Sum ? "sum" : reduce == ReduceKind::Max ? "max" : "min";
    case OpKind::Reshape: return "reshape";
    case OpKind::Transpose: return "transpose";
    case OpKind::BroadcastTo: return "broadcast_to";
    case OpKind::Slice: return "slice";
    case OpKind::Pad: return "pad";
    case OpKind::Cast: return "cast";
    case OpKind::StopGradient: return "stop_gradient";
    case OpKind::Floor: return "floor";
    case OpKind::Take: return "take";
    case OpKind::TakeAlong: return "take_along";
    case OpKind::TakeGrad: return "take_grad";
    case OpKind::TakeAlongGrad: return "take_along_grad";
    case OpKind::Concat: return "concat";
    case OpKind::Argmax: return "argmax";
    case OpKind::RandUniform: return "random_uniform";
    case OpKind::RandNormal: return "random_normal";
    case OpKind::KeySplit: return "key_split";
    case OpKind::ArgTopK: return "arg_top_k";
    case OpKind::Cumsum: return "cumsum";
    case OpKind::Scan: return "scan";
    case OpKind::While: return "while_loop";
    case OpKind::Cond: return "cond";
    case OpKind::Output: return "output";
    case OpKind::Placeholder: return "placeholder";
    case OpKind::Custom: return "custom_vjp";
    case OpKind::AllReduce: return "all_reduce";
    case OpKind::AttnFwd: return "attention";
    case OpKind::AttnBwd: return "attention_grad";
  }
  return "?";
}

bool Op::is_unary_elementwise() const {
  switch (kind) {
    case OpKind::Neg: case OpKind::Exp: case OpKind::Log: case OpKind::Sqrt: case OpKind::Sin:
    case OpKind::Cos: case OpKind::Tanh: case OpKind::Abs: case OpKind::Sign: case OpKind::Floor:
      return true;
    default: return false;
  }
}

bool Op::is_binary_elementwise() const {
  switch (kind) {
    case OpKind::Add: case OpKind::Sub: case OpKind::Mul: case OpKind::Div: case OpKind::Pow:
    case OpKind::Max: case OpKind::Min: case OpKind::Gt: case OpKind::Ge:
      return true;
    default: return false;
  }
}

// graph.rs:182-185
bool Op::int_ok() const {
  switch (kind) {
    case OpKind::Add: case OpKind::Sub: case OpKind::Mul: case OpKind::Gt: case OpKind::Ge:
    case OpKind::Where: case OpKind::Reshape: case OpKind::Transpose: case OpKind::BroadcastTo:
    case OpKind::Slice: case OpKind::Concat: case OpKind::Take: case OpKind::TakeAlong:
    case OpKind::Cast: case OpKind::StopGradient: case OpKind::Cumsum:
      return true;
    default: return false;
  }
}

bool Op::is_nonsmooth() const {
  switch (kind) {
    case OpKind::Abs: case OpKind::Sign: case OpKind::Floor: case OpKind::Max: case OpKind::Min:
    case OpKind::Gt: case OpKind::Ge: case OpKind::Where: case OpKind::Custom: case OpKind::ArgTopK:
    case OpKind::Cond:
      return true;
    case OpKind::Reduce: return reduce != ReduceKind::Sum;
    default: return false;
  }
}

static void key_vec(std::string& k, const char* tag, const std::vector<size_t>& v) {
  k += tag;
  k += '[';
  for (size_t x : v) {
    k += std::to_string(x);
    k += ',';
  }
  k += ']';
}

std::string Op::key() const {
  std::string k = std::to_string((int)kind);
  k += ':';
  k += std::to_string(index);
  key_vec(k, "s", shape);
  key_vec(k, "a", starts);
  key_vec(k, "o", stops);
  k += "d" + std::to_string((int)dtype) + (flag_a ? "A" : "a") + (flag_b ? "B" : "b") + "r" + std::to_string((int)reduce);
  if (value) {
    // Small constants only (callers skip large ones); NaN payloads compare equal like their
    // debug form does.
    key_vec(k, "cs", value->shape);
    k += "cd" + std::to_string((int)value->dtype());
    char b[32];
    for (size_t i = 0; i < value->n(); ++i) {
      double x = value->data.get(i);
      if (std::isnan(x)) {
        k += "nan,";
      } else {
        uint64_t bits;
        std::memcpy(&bits, &x, 8);
        snprintf(b, sizeof b, "%llx,", (unsigned long long)bits);
        k += b;
      }
    }
  }
  if (body) {
    char b[40];
    snprintf(b, sizeof b, "B%p", (void*)body.get());
    k += b;
  }
  if (body2) {
    char b[40];
    snprintf(b, sizeof b, "C%p", (void*)body2.get());
    k += b;
  }
  k += "n" + std::to_string(n_carry) + "," + std::to_string(n_x) + "," + std::to_string(length) + "," + std::to_string(max_iterations);
  k += "p" + std::to_string(placeholder);
  for (auto& r : rules) k += "r" + std::to_string(r.first) + "," + std::to_string(r.second);
  return k;
}

Json diag(const std::string& code, const std::string& severity, Json node, Json observation,
          const std::string& cause, const std::string& certainty) {
  Json d = Json::object();
  d["status"] = severity == "error" ? "validation_failed" : "warning";
  d["severity"] = severity;
  d["code"] = code;
  d["node"] = std::move(node);
  d["observation"] = std::move(observation);
  Json dg = Json::object();
  dg["cause"] = cause;
  dg["certainty"] = certainty;
  d["diagnosis"] = dg;
  return d;
}

bool broadcast_shapes(const std::vector<size_t>& a, const std::vector<size_t>& b, std::vector<size_t>* out) {
  size_t r = std::max(a.size(), b.size());
  std::vector<size_t> o(r, 0);
  for (size_t i = 0; i < r; ++i) {
    size_t x = i < a.size() ? a[a.size() - 1 - i] : 1;
    size_t y = i < b.size() ? b[b.size() - 1 - i] : 1;
    if (x != y && x != 1 && y != 1) return false;
    o[r - 1 - i] = std::max(x, y);
  }
  if (out) *out = std::move(o);
  return true;
}

static Json src_json(const std::shared_ptr<const std::string>& s) {
  return s ? Json(*s) : Json(nullptr);
}

// graph.rs:233-248
Json Graph::node_json(uint32_t id) const {
  const Node& n = nodes[id];
  Json v = Json::object();
  v["id"] = id;
  v["operation"] = n.op.name();
  v["source"] = src_json(n.source);
  v["role"] = n.origin ? "backward" : "forward";
  if (n.origin) {
    const Node& f = nodes[*n.origin];
    Json fw = Json::object();
    fw["id"] = *n.origin;
    fw["operation"] = f.op.name();
    fw["source"] = src_json(f.source);
    v["forward_node"] = fw;
  }
  return v;
}

Json Graph::pending_json(const Op& op) const {
  Json v = Json::object();
  v["id"] = nullptr;
  v["operation"] = op.name();
  v["source"] = src_json(cur_source);
  v["role"] = "forward";
  return v;
}

void Graph::static_err(const std::string& code, const Op& op, Json obs, const std::string& cause) const {
  throw DiagError(diag(code, "error", pending_json(op), std::move(obs), cause, "verified"));
}

uint32_t Graph::push(Op op, std::vector<uint32_t> inputs, std::vector<size_t> shape, DType d) {
  Node n;
  n.op = std::move(op);
  n.inputs = std::move(inputs);
  n.shape = std::move(shape);
  n.dtype = d;
  n.source = cur_source;
  n.origin = cur_origin;
  nodes.push_back(std::move(n));
  return (uint32_t)(nodes.size() - 1);
}

uint32_t Graph::input(const std::vector<size_t>& shape, DType d) {
  Op o = Op::make(OpKind::Input);
  o.index = n_inputs++;
  return push(std::move(o), {}, shape, d);
}

uint32_t Graph::placeholder(const std::vector<size_t>& shape, DType d) {
  return push(Op::make(OpKind::Placeholder), {}, shape, d);
}

uint32_t Graph::constant(Tensor t) { return constant(std::make_shared<const Tensor>(std::move(t))); }

uint32_t Graph::constant(TensorP t) {
  Op o = Op::make(OpKind::Const);
  auto s = t->shape;
  auto d = t->dtype();
  o.value = std::move(t);
  return push(std::move(o), {}, s, d);
}

static Json shapes_json(const std::vector<std::vector<size_t>>& s) {
  Json a = Json::array();
  for (auto& x : s) a.push(Json(x));
  return a;
}

uint32_t Graph::add(Op op, const std::vector<uint32_t>& inputs) {
  for (uint32_t i : inputs) {
    if (i >= nodes.size()) {
      Json o = Json::object();
      o["input"] = i;
      static_err("INVALID_NODE_REF", op, o, "unknown_node_id");
    }
  }
  size_t arity;
  switch (op.kind) {
    case OpKind::Input: case OpKind::Const: case OpKind::Placeholder: arity = 0; break;
    case OpKind::Where: arity = 3; break;
    case OpKind::MatMul: case OpKind::MatMulT: case OpKind::Take: case OpKind::TakeAlong:
    case OpKind::TakeGrad: case OpKind::TakeAlongGrad: arity = 2; break;
    case OpKind::Concat: arity = std::max<size_t>(inputs.size(), 1); break;
    // With a third attribute (heads) q, k, v come as one packed tensor: (qkv, mask) and
    // (qkv, mask, fwd, dO).
    case OpKind::AttnFwd: arity = op.value && op.value->n() == 3 ? 2 : 4; break;
    case OpKind::AttnBwd: arity = op.value && op.value->n() == 3 ? 4 : 6; break;
    default:
      if (op.is_control_flow()) arity = inputs.size();
      else if (op.is_binary_elementwise()) arity = 2;
      else arity = 1;
  }
  if (inputs.size() != arity) {
    Json o = Json::object();
    o["expected"] = arity;
    o["actual"] = inputs.size();
    static_err("ARITY_MISMATCH", op, o, "wrong_input_count");
  }
  if (op.is_control_flow()) {
    check_control_flow(op, inputs);
    return push(std::move(op), inputs, {}, DType::F32);
  }
  if (op.kind == OpKind::Output) {
    auto s = op.shape;
    auto d = op.dtype;
    return push(std::move(op), inputs, s, d);
  }
  std::vector<DType> dts;
  for (uint32_t i : inputs) dts.push_back(dtype(i));
  bool indexes = op.kind == OpKind::Take || op.kind == OpKind::TakeAlong || op.kind == OpKind::TakeGrad || op.kind == OpKind::TakeAlongGrad;
  if (indexes && dts[1] != DType::I32) {
    Json o = Json::object();
    o["index_dtype"] = dtype_name(dts[1]);
    static_err("DTYPE_MISMATCH", op, o, "index_must_be_int32");
  }
  bool random = op.kind == OpKind::RandUniform || op.kind == OpKind::RandNormal || op.kind == OpKind::KeySplit;
  if (random && (dts[0] != DType::I32 || shape(inputs[0]) != std::vector<size_t>{2})) {
    Json o = Json::object();
    o["key_shape"] = Json(shape(inputs[0]));
    o["key_dtype"] = dtype_name(dts[0]);
    static_err("INVALID_KEY", op, o, "key_must_be_int32_of_shape_2");
  }
  if (!indexes && !random && op.kind != OpKind::Cast) {
    for (size_t k = 1; k < dts.size(); ++k) {
      if (dts[k] != dts[k - 1]) {
        Json names = Json::array();
        for (auto d : dts) names.push(dtype_name(d));
        Json o = Json::object();
        o["input_dtypes"] = names;
        static_err("DTYPE_MISMATCH", op, o, "implicit_promotion_not_allowed");
      }
    }
  }
  if (!random && op.kind != OpKind::Argmax && op.kind != OpKind::ArgTopK && dts[0] == DType::I32 && !op.int_ok()) {
    Json o = Json::object();
    o["dtype"] = "int32";
    static_err("UNSUPPORTED_DTYPE", op, o, "operation_is_float_only_cast_first");
  }
  DType dt;
  switch (op.kind) {
    case OpKind::Cast: dt = op.dtype; break;
    case OpKind::RandUniform: case OpKind::RandNormal: dt = op.dtype; break;
    case OpKind::KeySplit: case OpKind::Argmax: case OpKind::ArgTopK: dt = DType::I32; break;
    default: dt = dts[0];
  }
  std::vector<std::vector<size_t>> shapes;
  for (uint32_t i : inputs) shapes.push_back(nodes[i].shape);

  if (op.kind == OpKind::Where) {
    // Materializing the broadcast keeps the Where kernel same-shape only (graph.rs:368-379).
    std::vector<size_t> target;
    bool ok = true;
    for (auto& s : shapes) {
      std::vector<size_t> next;
      if (!broadcast_shapes(target, s, &next)) {
        ok = false;
        break;
      }
      target = next;
    }
    if (!ok) {
      Json o = Json::object();
      o["input_shapes"] = shapes_json(shapes);
      static_err("SHAPE_MISMATCH", op, o, "incompatible_broadcast");
    }
    std::vector<uint32_t> ids;
    for (size_t k = 0; k < inputs.size(); ++k) {
      if (shapes[k] == target) {
        ids.push_back(inputs[k]);
      } else {
        Op b = Op::make(OpKind::BroadcastTo);
        b.shape = target;
        ids.push_back(add(std::move(b), {inputs[k]}));
      }
    }
    return push(std::move(op), ids, target, dt);
  }
  auto sh = infer(op, shapes);
  return push(std::move(op), inputs, std::move(sh), dt);
}

std::vector<size_t> Graph::infer(const Op& op, const std::vector<std::vector<size_t>>& s) const {
  if (op.is_unary_elementwise() || op.kind == OpKind::Cast || op.kind == OpKind::StopGradient) return s[0];
  if (op.is_binary_elementwise()) {
    std::vector<size_t> out;
    if (!broadcast_shapes(s[0], s[1], &out)) {
      Json o = Json::object();
      o["lhs_shape"] = Json(s[0]);
      o["rhs_shape"] = Json(s[1]);
      static_err("SHAPE_MISMATCH", op, o, "incompatible_broadcast");
    }
    return out;
  }
  switch (op.kind) {
    case OpKind::MatMul: {
      const auto &a = s[0], &b = s[1];
      if (a.empty() || b.empty()) {
        Json o = Json::object();
        o["lhs_shape"] = Json(a);
        o["rhs_shape"] = Json(b);
        o["minimum_rank"] = 1;
        static_err("UNSUPPORTED_RANK", op, o, "matmul_of_scalar");
      }
      size_t ka = a.back();
      size_t kb = b.size() >= 2 ? b[b.size() - 2] : b[0];
      if (ka != kb) {
        Json o = Json::object();
        o["lhs_shape"] = Json(a);
        o["rhs_shape"] = Json(b);
        o["lhs_inner"] = ka;
        o["rhs_inner"] = kb;
        static_err("SHAPE_MISMATCH", op, o, "matmul_inner_dimension_mismatch");
      }
      std::vector<size_t> ba(a.begin(), a.end() - std::min<size_t>(2, a.size()));
      std::vector<size_t> bb(b.begin(), b.end() - std::min<size_t>(2, b.size()));
      std::vector<size_t> out;
      if (!broadcast_shapes(ba, bb, &out)) {
        Json o = Json::object();
        o["lhs_shape"] = Json(a);
        o["rhs_shape"] = Json(b);
        static_err("SHAPE_MISMATCH", op, o, "matmul_batch_dimensions_incompatible");
      }
      if (a.size() >= 2) out.push_back(a[a.size() - 2]);
      if (b.size() >= 2) out.push_back(b.back());
      return out;
    }
    case OpKind::MatMulT: {
      auto view = [](std::vector<size_t> t, bool flip) {
        if (flip) std::swap(t[t.size() - 2], t[t.size() - 1]);
        return t;
      };
      return infer(Op::make(OpKind::MatMul), {view(s[0], op.flag_a), view(s[1], op.flag_b)});
    }
    case OpKind::Take: {
      size_t axis = op.index;
      if (axis >= s[0].size() || s[0][axis] == 0) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        o["axis"] = axis;
        static_err("INVALID_AXIS", op, o, "axis_out_of_range_or_empty");
      }
      std::vector<size_t> out(s[0].begin(), s[0].begin() + axis);
      out.insert(out.end(), s[1].begin(), s[1].end());
      out.insert(out.end(), s[0].begin() + axis + 1, s[0].end());
      return out;
    }
    case OpKind::TakeAlong: {
      bool ok = !s[0].empty() && s[0].size() == s[1].size() &&
                std::equal(s[0].begin(), s[0].end() - 1, s[1].begin()) && s[0].back() > 0;
      if (!ok) {
        Json o = Json::object();
        o["values_shape"] = Json(s[0]);
        o["index_shape"] = Json(s[1]);
        static_err("SHAPE_MISMATCH", op, o, "take_along_requires_matching_batch_dimensions");
      }
      return s[1];
    }
    case OpKind::TakeGrad: case OpKind::TakeAlongGrad: return op.shape;
    case OpKind::Concat: {
      size_t rank = s[0].size();
      size_t axis = op.index;
      bool ok = axis < rank;
      for (auto& t : s) {
        if (!ok) break;
        if (t.size() != rank) { ok = false; break; }
        for (size_t d = 0; d < rank; ++d)
          if (d != axis && t[d] != s[0][d]) ok = false;
      }
      if (!ok) {
        Json o = Json::object();
        o["input_shapes"] = shapes_json(s);
        o["axis"] = axis;
        static_err("SHAPE_MISMATCH", op, o, "concat_shapes_differ_off_axis");
      }
      std::vector<size_t> out = s[0];
      out[axis] = 0;
      for (auto& t : s) out[axis] += t[axis];
      return out;
    }
    case OpKind::ArgTopK: {
      size_t v = s[0].empty() ? 0 : s[0].back();
      if (op.index == 0 || op.index > v) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        o["k"] = op.index;
        static_err("INVALID_AXIS", op, o, "k_must_be_between_one_and_the_last_axis_size");
      }
      std::vector<size_t> out = s[0];
      out.back() = op.index;
      return out;
    }
    case OpKind::Cumsum: {
      if (s[0].empty()) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        static_err("INVALID_AXIS", op, o, "cumsum_needs_at_least_one_axis");
      }
      return s[0];
    }
    case OpKind::Argmax: {
      if (s[0].empty() || s[0].back() == 0) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        static_err("INVALID_AXIS", op, o, "argmax_needs_a_nonempty_last_axis");
      }
      return std::vector<size_t>(s[0].begin(), s[0].end() - 1);
    }
    case OpKind::RandUniform: case OpKind::RandNormal: return op.shape;
    case OpKind::KeySplit: return {op.index, 2};
    case OpKind::Custom: case OpKind::AllReduce: return s[0];
    case OpKind::AttnFwd: case OpKind::AttnBwd: {
      if (op.value && op.value->n() == 3) {
        // Packed: qkv (B, T, 3, H, d) with H the third attribute, mask (T, T); AttnBwd also the
        // forward's packed output (B, H, T, d + 2) and dO (B, T, H, d). AttnFwd gives
        // (B, H, T, d + 2), AttnBwd the gradient of qkv, (B, T, 3, H, d).
        const auto& x = s[0];
        const size_t heads = (size_t)op.value->data.get(2);
        bool ok = x.size() == 5 && x[2] == 3 && x[3] == heads && heads > 0 && s[1] == std::vector<size_t>{x[1], x[1]};
        if (ok && op.kind == OpKind::AttnBwd)
          ok = s[2] == std::vector<size_t>{x[0], heads, x[1], x[4] + 2} && s[3] == std::vector<size_t>{x[0], x[1], heads, x[4]};
        if (!ok) {
          Json o = Json::object();
          o["input_shapes"] = shapes_json(s);
          static_err("SHAPE_MISMATCH", op, o, "attention_operands_do_not_fit");
        }
        if (op.kind == OpKind::AttnBwd) return x;
        return {x[0], heads, x[1], x[4] + 2};
      }
      // q (..., T, d), k (..., T, d), v (..., T, dv) with the same leading extents, mask (T, T);
      // AttnBwd also the forward's packed output (..., T, dv + 2) and dO (..., T, dv).
      const auto &q = s[0], &k = s[1], &v = s[2], &m = s[3];
      size_t r = q.size();
      bool ok = r >= 2 && k.size() == r && v.size() == r && m.size() == 2;
      for (size_t i = 0; ok && i + 2 < r; ++i) ok = k[i] == q[i] && v[i] == q[i];
      size_t t = ok ? q[r - 2] : 0, d = ok ? q[r - 1] : 0, dv = ok ? v[r - 1] : 0;
      ok = ok && k[r - 2] == t && v[r - 2] == t && k[r - 1] == d && m[0] == t && m[1] == t;
      if (ok && op.kind == OpKind::AttnBwd) {
        std::vector<size_t> st = q, dout = v;
        st[r - 1] = dv + 2;
        ok = s[4] == st && s[5] == dout;
      }
      if (!ok || !op.value || op.value->n() != 2) {
        Json o = Json::object();
        o["input_shapes"] = shapes_json(s);
        static_err("SHAPE_MISMATCH", op, o, "attention_operands_do_not_fit");
      }
      std::vector<size_t> out = q;
      out[r - 1] = op.kind == OpKind::AttnFwd ? dv + 2 : 2 * d + dv;
      return out;
    }
    case OpKind::Reduce: {
      size_t r = s[0].size();
      std::vector<bool> seen(r, false);
      for (size_t a : op.shape) {
        if (a >= r || seen[a]) {
          Json o = Json::object();
          o["shape"] = Json(s[0]);
          o["axes"] = Json(op.shape);
          static_err("INVALID_AXIS", op, o, "axis_out_of_range_or_duplicate");
        }
        seen[a] = true;
      }
      for (size_t a : op.shape) {
        if (s[0][a] == 0) {
          Json o = Json::object();
          o["shape"] = Json(s[0]);
          o["axes"] = Json(op.shape);
          static_err("INVALID_AXIS", op, o, "reduction_over_empty_axis");
        }
      }
      std::vector<size_t> out;
      for (size_t i = 0; i < r; ++i) {
        if (seen[i]) {
          if (op.flag_a) out.push_back(1);
        } else {
          out.push_back(s[0][i]);
        }
      }
      return out;
    }
    case OpKind::Reshape: {
      if (product(op.shape) != product(s[0])) {
        Json o = Json::object();
        o["input_shape"] = Json(s[0]);
        o["target_shape"] = Json(op.shape);
        static_err("SHAPE_MISMATCH", op, o, "reshape_element_count_mismatch");
      }
      return op.shape;
    }
    case OpKind::Transpose: {
      std::vector<size_t> sorted = op.shape;
      std::sort(sorted.begin(), sorted.end());
      bool ok = sorted.size() == s[0].size();
      for (size_t i = 0; ok && i < sorted.size(); ++i) ok = sorted[i] == i;
      if (!ok) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        o["perm"] = Json(op.shape);
        static_err("INVALID_AXIS", op, o, "invalid_permutation");
      }
      std::vector<size_t> out;
      for (size_t p : op.shape) out.push_back(s[0][p]);
      return out;
    }
    case OpKind::BroadcastTo: {
      std::vector<size_t> out;
      if (!broadcast_shapes(s[0], op.shape, &out) || out != op.shape) {
        Json o = Json::object();
        o["input_shape"] = Json(s[0]);
        o["target_shape"] = Json(op.shape);
        static_err("SHAPE_MISMATCH", op, o, "incompatible_broadcast");
      }
      return op.shape;
    }
    case OpKind::Slice: {
      size_t r = s[0].size();
      bool ok = op.starts.size() == r && op.stops.size() == r;
      for (size_t i = 0; ok && i < r; ++i) ok = op.starts[i] <= op.stops[i] && op.stops[i] <= s[0][i];
      if (!ok) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        o["starts"] = Json(op.starts);
        o["stops"] = Json(op.stops);
        static_err("INVALID_SLICE", op, o, "slice_out_of_bounds");
      }
      std::vector<size_t> out;
      for (size_t i = 0; i < r; ++i) out.push_back(op.stops[i] - op.starts[i]);
      return out;
    }
    case OpKind::Pad: {
      size_t r = s[0].size();
      bool ok = op.starts.size() == r && op.shape.size() == r;
      for (size_t i = 0; ok && i < r; ++i) ok = op.starts[i] + s[0][i] <= op.shape[i];
      if (!ok) {
        Json o = Json::object();
        o["shape"] = Json(s[0]);
        o["starts"] = Json(op.starts);
        o["target_shape"] = Json(op.shape);
        static_err("INVALID_SLICE", op, o, "pad_out_of_bounds");
      }
      return op.shape;
    }
    default:
      throw std::logic_error("op without inputs reached infer");
  }
}

// graph.rs:524-558
void Graph::check_control_flow(const Op& op, const std::vector<uint32_t>& inputs) const {
  auto expect = [&](const Body& body, const std::vector<uint32_t>& args, size_t st_lo, size_t st_hi, size_t length) {
    std::vector<std::pair<std::vector<size_t>, DType>> want(body.graph.n_inputs, {{}, DType::F32});
    for (auto& n : body.graph.nodes)
      if (n.op.kind == OpKind::Input) want[n.op.index] = {n.shape, n.dtype};
    bool ok = want.size() == args.size();
    for (size_t k = 0; ok && k < args.size(); ++k) {
      const auto& have = shape(args[k]);
      bool elem;
      if (k >= st_lo && k < st_hi) {
        elem = !have.empty() && have[0] == length && std::vector<size_t>(have.begin() + 1, have.end()) == want[k].first;
      } else {
        elem = have == want[k].first;
      }
      ok = elem && dtype(args[k]) == want[k].second;
    }
    if (!ok) {
      Json o = Json::object();
      Json w = Json::array(), h = Json::array();
      for (auto& x : want) w.push(Json(x.first));
      for (auto a : args) h.push(Json(shape(a)));
      o["body_inputs"] = w;
      o["given_inputs"] = h;
      static_err("CONTROL_FLOW_SHAPE_MISMATCH", op, o, "inputs_differ_from_the_traced_body");
    }
  };
  switch (op.kind) {
    case OpKind::Scan: expect(*op.body, inputs, op.n_carry, op.n_carry + op.n_x, op.length); break;
    case OpKind::While:
      expect(*op.body, inputs, 0, 0, 0);
      expect(*op.body2, inputs, 0, 0, 0);
      break;
    case OpKind::Cond: {
      std::vector<uint32_t> rest(inputs.begin() + 1, inputs.end());
      expect(*op.body, rest, 0, 0, 0);
      expect(*op.body2, rest, 0, 0, 0);
      break;
    }
    default: throw std::logic_error("only control flow is checked here");
  }
}

std::vector<bool> Graph::reachable(const std::vector<uint32_t>& outputs) const {
  std::vector<bool> keep(nodes.size(), false);
  for (auto o : outputs) keep[o] = true;
  for (size_t i = nodes.size(); i-- > 0;)
    if (keep[i])
      for (auto x : nodes[i].inputs) keep[x] = true;
  return keep;
}

// graph.rs:577-608
Graph Graph::to_f64() const {
  Graph g = *this;
  auto widen = [](const BodyP& b) { return Body::make(b->graph.to_f64(), b->outputs); };
  for (auto& n : g.nodes) {
    switch (n.op.kind) {
      case OpKind::Scan: n.op.body = widen(n.op.body); break;
      case OpKind::While:
      case OpKind::Cond:
        n.op.body = widen(n.op.body);
        n.op.body2 = widen(n.op.body2);
        break;
      case OpKind::Output:
        if (n.op.dtype != DType::I32) n.op.dtype = DType::F64;
        break;
      default: break;
    }
    if (n.dtype == DType::I32) continue;
    n.dtype = DType::F64;
    switch (n.op.kind) {
      case OpKind::Const:
        n.op.value = std::make_shared<const Tensor>(Tensor::from_f64(DType::F64, n.op.value->shape, n.op.value->data.to_f64()));
        break;
      case OpKind::Cast: n.op.dtype = DType::F64; break;
      case OpKind::RandUniform: case OpKind::RandNormal: n.op.dtype = DType::F64; break;
      default: break;
    }
  }
  return g;
}

// graph.rs:27-32
BodyP Body::make(Graph g, std::vector<uint32_t> outputs) {
  auto b = std::make_shared<Body>();
  OptResult r = optimize(g, outputs);
  b->opt = std::move(r.graph);
  b->opt_outputs = std::move(r.outputs);
  b->fast = std::make_shared<Plan>(Plan::build_fused(b->opt, b->opt_outputs, Fuse::DEFAULT()));
  b->reference = std::make_shared<Plan>(Plan::build(g, outputs, false));
  b->graph = std::move(g);
  b->outputs = std::move(outputs);
  return b;
}

std::shared_ptr<Plan> Body::plan_for(const Fuse& f) {
  std::string k = f.key();
  std::lock_guard<std::mutex> lk(mu_);
  if (k == Fuse::DEFAULT().key()) return fast;
  for (auto& c : cache_)
    if (c.first == k) return c.second;
  auto p = std::make_shared<Plan>(Plan::build_fused(opt, opt_outputs, f));
  cache_.emplace_back(k, p);
  return p;
}

}  // namespace rg
