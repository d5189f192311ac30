// Reverse-mode VJP rules; each rule restates the matching arm of src/autodiff.rs:328-557.
// Rule forms are kept node for node, since they decide the rounding of every gradient.
#include "autodiff.h"

#include <algorithm>
#include <map>
#include <stdexcept>

namespace rg {

namespace {

uint32_t add1(Graph& g, OpKind k, uint32_t a) { return g.add(Op::make(k), {a}); }
uint32_t add2(Graph& g, OpKind k, uint32_t a, uint32_t b) { return g.add(Op::make(k), {a, b}); }
uint32_t reshape(Graph& g, std::vector<size_t> s, uint32_t x) {
  Op o = Op::make(OpKind::Reshape);
  o.shape = std::move(s);
  return g.add(std::move(o), {x});
}
uint32_t reduce_sum(Graph& g, std::vector<size_t> axes, bool keepdims, uint32_t x) {
  Op o = Op::make(OpKind::Reduce);
  o.reduce = ReduceKind::Sum;
  o.shape = std::move(axes);
  o.flag_a = keepdims;
  return g.add(std::move(o), {x});
}

// autodiff.rs:7-16
uint32_t unbroadcast(Graph& g, uint32_t ct, const std::vector<size_t>& target) {
  auto shape = g.shape(ct);
  if (shape == target) return ct;
  size_t lead = shape.size() - target.size();
  std::vector<size_t> axes;
  for (size_t i = 0; i < shape.size(); ++i)
    if (i < lead || (target[i - lead] == 1 && shape[i] != 1)) axes.push_back(i);
  uint32_t summed = reduce_sum(g, axes, true, ct);
  return reshape(g, target, summed);
}

bool blocks_gradient(const Op& op) {
  switch (op.kind) {
    case OpKind::StopGradient: case OpKind::Sign: case OpKind::Gt: case OpKind::Ge: case OpKind::Floor:
    case OpKind::Argmax: case OpKind::RandUniform: case OpKind::RandNormal: case OpKind::KeySplit:
    case OpKind::Placeholder: case OpKind::ArgTopK:
      return true;
    default: return false;
  }
}

struct Vjp {
  Graph graph;
  std::vector<uint32_t> grads;
  std::vector<size_t> float_in, float_out;
};

// autodiff.rs:32-61
Vjp vjp_graph(const Body& body) {
  Graph g = body.graph;
  g.grads.clear();
  g.notes.clear();
  size_t n_in = g.n_inputs;
  std::vector<uint32_t> inputs(n_in, 0);
  for (size_t id = 0; id < g.nodes.size(); ++id)
    if (g.nodes[id].op.kind == OpKind::Input) inputs[g.nodes[id].op.index] = (uint32_t)id;
  Vjp v;
  for (size_t k = 0; k < n_in; ++k)
    if (g.dtype(inputs[k]) != DType::I32) v.float_in.push_back(k);
  for (size_t k = 0; k < body.outputs.size(); ++k)
    if (body.output_dtype(k) != DType::I32) v.float_out.push_back(k);
  DType d = v.float_in.empty() ? DType::F32 : g.dtype(inputs[v.float_in[0]]);
  uint32_t total = g.scalar(d, 0.0);
  for (size_t k : v.float_out) {
    uint32_t o = body.outputs[k];
    uint32_t ct = g.input(body.output_shape(k), body.output_dtype(k));
    uint32_t m = add2(g, OpKind::Mul, o, ct);
    std::vector<size_t> axes;
    for (size_t a = 0; a < g.shape(m).size(); ++a) axes.push_back(a);
    uint32_t sum = reduce_sum(g, axes, false, m);
    if (g.dtype(sum) != d) {
      Op c = Op::make(OpKind::Cast);
      c.dtype = d;
      sum = g.add(std::move(c), {sum});
    }
    total = add2(g, OpKind::Add, total, sum);
  }
  std::vector<uint32_t> wrts;
  for (size_t k : v.float_in) wrts.push_back(inputs[k]);
  v.grads = grad(g, total, wrts);
  g.notes.clear();
  g.grads.clear();
  v.graph = std::move(g);
  return v;
}

uint32_t zeros_for(Graph& g, const std::vector<size_t>& shape, DType d) { return g.constant(Tensor::full(d, shape, 0.0)); }

uint32_t body_input(const Body& body, size_t k) {
  for (size_t i = 0; i < body.graph.nodes.size(); ++i)
    if (body.graph.nodes[i].op.kind == OpKind::Input && body.graph.nodes[i].op.index == k) return (uint32_t)i;
  throw std::logic_error("every input exists");
}

uint32_t output_of(Graph& g, uint32_t node, size_t index, std::vector<size_t> shape, DType d) {
  Op o = Op::make(OpKind::Output);
  o.index = index;
  o.shape = std::move(shape);
  o.dtype = d;
  return g.add(std::move(o), {node});
}

using Pairs = std::vector<std::pair<uint32_t, uint32_t>>;

// autodiff.rs:68-231
Pairs vjp_control(Graph& g, size_t i, const std::map<size_t, uint32_t>& cots, const std::vector<bool>& rel) {
  Node node = g.nodes[i];
  Pairs out;
  if (node.op.kind == OpKind::While) {
    Json obs = Json::object();
    obs["alternative"] = "rg.scan with a fixed length";
    throw DiagError(diag("GRAD_THROUGH_WHILE", "error", g.node_json((uint32_t)i), obs, "iteration_count_is_a_runtime_value", "verified"));
  }
  if (node.op.kind == OpKind::Cond) {
    const Body& then_body = *node.op.body;
    Vjp t = vjp_graph(then_body);
    Vjp e = vjp_graph(*node.op.body2);
    auto float_in = t.float_in;
    auto float_out = t.float_out;
    BodyP tb = Body::make(std::move(t.graph), t.grads);
    BodyP eb = Body::make(std::move(e.graph), e.grads);
    std::vector<uint32_t> ins = node.inputs;
    for (size_t k : float_out) {
      auto it = cots.find(k);
      ins.push_back(it != cots.end() ? it->second : zeros_for(g, then_body.output_shape(k), then_body.output_dtype(k)));
    }
    Op c = Op::make(OpKind::Cond);
    c.body = tb;
    c.body2 = eb;
    uint32_t cond = g.add(std::move(c), ins);
    for (size_t j = 0; j < float_in.size(); ++j) {
      uint32_t target = node.inputs[float_in[j] + 1];
      if (rel[target]) out.emplace_back(target, output_of(g, cond, j, g.shape(target), g.dtype(target)));
    }
    return out;
  }
  // Scan
  const Body& body = *node.op.body;
  size_t c = node.op.n_carry, x = node.op.n_x, len = node.op.length;
  size_t m = body.graph.n_inputs - c - x;
  size_t n_y = body.outputs.size() - c;
  Vjp v = vjp_graph(body);
  Graph& r = v.graph;
  std::vector<size_t> fc, fy, g_x, g_cap;
  for (size_t k : v.float_out) (k < c ? fc : fy).push_back(k);
  for (size_t j = 0; j < v.float_in.size(); ++j) {
    if (v.float_in[j] >= c && v.float_in[j] < c + x) g_x.push_back(j);
    if (v.float_in[j] >= c + x) g_cap.push_back(j);
  }
  size_t n_ct = fc.size(), n_acc = g_cap.size();
  bool any_hist = false;
  for (size_t k : fc) any_hist = any_hist || cots.count(c + n_y + k);
  std::vector<size_t> hist = any_hist ? fc : std::vector<size_t>{};
  size_t n_orig = c + x + m;
  auto renumber = [&](size_t k) -> size_t {
    if (k < c) return n_ct + n_acc + k;
    if (k < c + x) return n_ct + n_acc + c + (k - c);
    if (k < n_orig) return n_ct + n_acc + c + x + fy.size() + hist.size() + (k - c - x);
    if (k - n_orig < n_ct) return k - n_orig;
    return n_ct + n_acc + c + x + (k - n_orig - n_ct);
  };
  for (auto& nd : r.nodes)
    if (nd.op.kind == OpKind::Input) nd.op.index = renumber(nd.op.index);
  std::vector<uint32_t> acc_inputs;
  auto push_input = [&](size_t index, const std::vector<size_t>& s, DType d) {
    Node nd;
    nd.op = Op::make(OpKind::Input);
    nd.op.index = index;
    nd.shape = s;
    nd.dtype = d;
    r.nodes.push_back(std::move(nd));
    r.n_inputs += 1;
    return (uint32_t)(r.nodes.size() - 1);
  };
  for (size_t a = 0; a < g_cap.size(); ++a) {
    uint32_t id = v.grads[g_cap[a]];
    acc_inputs.push_back(push_input(n_ct + a, r.shape(id), r.dtype(id)));
  }
  std::vector<uint32_t> outs;
  for (size_t k : fc) {
    size_t j = std::find(v.float_in.begin(), v.float_in.end(), k) - v.float_in.begin();
    uint32_t gradient = v.grads[j];
    auto pos = std::find(hist.begin(), hist.end(), k);
    if (pos != hist.end()) {
      size_t a = pos - hist.begin();
      uint32_t saved = push_input(n_ct + n_acc + c + x + fy.size() + a, r.shape(gradient), r.dtype(gradient));
      gradient = add2(r, OpKind::Add, gradient, saved);
    }
    outs.push_back(gradient);
  }
  for (size_t a = 0; a < g_cap.size(); ++a) outs.push_back(add2(r, OpKind::Add, acc_inputs[a], v.grads[g_cap[a]]));
  for (size_t j : g_x) outs.push_back(v.grads[j]);
  BodyP reverse_body = Body::make(std::move(r), outs);

  std::vector<uint32_t> ins;
  for (size_t k : fc) {
    auto it = cots.find(k);
    ins.push_back(it != cots.end() ? it->second : zeros_for(g, body.output_shape(k), body.output_dtype(k)));
  }
  for (size_t j : g_cap) {
    uint32_t target = node.inputs[v.float_in[j]];
    ins.push_back(zeros_for(g, g.shape(target), g.dtype(target)));
  }
  for (size_t k = 0; k < c; ++k) {
    std::vector<size_t> s{len};
    const auto& bs = body.graph.shape(body_input(body, k));
    s.insert(s.end(), bs.begin(), bs.end());
    ins.push_back(output_of(g, (uint32_t)i, c + n_y + k, s, body.graph.dtype(body_input(body, k))));
  }
  ins.insert(ins.end(), node.inputs.begin() + c, node.inputs.begin() + c + x);
  for (size_t k : fy) {
    std::vector<size_t> s{len};
    s.insert(s.end(), body.output_shape(k).begin(), body.output_shape(k).end());
    auto it = cots.find(k);
    ins.push_back(it != cots.end() ? it->second : zeros_for(g, s, body.output_dtype(k)));
  }
  for (size_t k : hist) {
    std::vector<size_t> s{len};
    const auto& bs = body.graph.shape(body_input(body, k));
    s.insert(s.end(), bs.begin(), bs.end());
    auto it = cots.find(c + n_y + k);
    ins.push_back(it != cots.end() ? it->second : zeros_for(g, s, body.graph.dtype(body_input(body, k))));
  }
  ins.insert(ins.end(), node.inputs.begin() + c + x, node.inputs.end());
  Op sc = Op::make(OpKind::Scan);
  sc.body = reverse_body;
  sc.n_carry = n_ct + n_acc;
  sc.n_x = c + x + fy.size() + hist.size();
  sc.length = len;
  sc.flag_a = !node.op.flag_a;
  uint32_t back = g.add(std::move(sc), ins);
  for (size_t a = 0; a < fc.size(); ++a) {
    uint32_t target = node.inputs[fc[a]];
    if (rel[target]) out.emplace_back(target, output_of(g, back, a, g.shape(target), g.dtype(target)));
  }
  for (size_t a = 0; a < g_cap.size(); ++a) {
    uint32_t target = node.inputs[v.float_in[g_cap[a]]];
    if (rel[target]) out.emplace_back(target, output_of(g, back, n_ct + a, g.shape(target), g.dtype(target)));
  }
  for (size_t a = 0; a < g_x.size(); ++a) {
    uint32_t target = node.inputs[v.float_in[g_x[a]]];
    if (rel[target]) out.emplace_back(target, output_of(g, back, n_ct + n_acc + a, g.shape(target), g.dtype(target)));
  }
  return out;
}

// Transposes the last two axes.
uint32_t swap_last(Graph& g, uint32_t v) {
  size_t r = g.shape(v).size();
  Op o = Op::make(OpKind::Transpose);
  for (size_t k = 0; k < r; ++k) o.shape.push_back(k);
  std::swap(o.shape[r - 2], o.shape[r - 1]);
  return g.add(std::move(o), {v});
}

// autodiff.rs:328-557
Pairs vjp(Graph& g, size_t i, uint32_t ct, const std::vector<bool>& rel) {
  Node node = g.nodes[i];
  uint32_t me = (uint32_t)i;
  DType d = node.dtype;
  uint32_t x = node.inputs.empty() ? 0 : node.inputs[0];
  uint32_t y = node.inputs.size() > 1 ? node.inputs[1] : 0;
  Pairs out;

  // Unary rules: dy/dx times the cotangent.
  int have_factor = 1;
  uint32_t f = 0;
  switch (node.op.kind) {
    case OpKind::Exp: f = me; break;
    case OpKind::Cos: f = add1(g, OpKind::Neg, add1(g, OpKind::Sin, x)); break;
    case OpKind::Sin: f = add1(g, OpKind::Cos, x); break;
    case OpKind::Tanh: {
      uint32_t one = g.scalar(d, 1.0);
      uint32_t sq = add2(g, OpKind::Mul, me, me);
      f = add2(g, OpKind::Sub, one, sq);
      break;
    }
    case OpKind::Abs: f = add1(g, OpKind::Sign, x); break;
    default: have_factor = 0;
  }
  if (have_factor) {
    out.emplace_back(x, add2(g, OpKind::Mul, ct, f));
    return out;
  }

  switch (node.op.kind) {
    case OpKind::Input: case OpKind::Const: case OpKind::StopGradient: case OpKind::Sign: case OpKind::Gt:
    case OpKind::Ge:
      break;
    case OpKind::Neg: out.emplace_back(x, add1(g, OpKind::Neg, ct)); break;
    case OpKind::Log: out.emplace_back(x, add2(g, OpKind::Div, ct, x)); break;
    case OpKind::Sqrt: {
      uint32_t two = g.scalar(d, 2.0);
      uint32_t denom = add2(g, OpKind::Mul, two, me);
      out.emplace_back(x, add2(g, OpKind::Div, ct, denom));
      break;
    }
    case OpKind::Add: case OpKind::Sub: case OpKind::Mul: case OpKind::Div: case OpKind::Pow: case OpKind::Max:
    case OpKind::Min: {
      auto sx = g.shape(x), sy = g.shape(y);
      OpKind k = node.op.kind;
      if (rel[x]) {
        uint32_t c;
        switch (k) {
          case OpKind::Add: case OpKind::Sub: c = ct; break;
          case OpKind::Mul: c = add2(g, OpKind::Mul, ct, y); break;
          case OpKind::Div: c = add2(g, OpKind::Div, ct, y); break;
          case OpKind::Pow: {
            uint32_t one = g.scalar(d, 1.0);
            uint32_t e = add2(g, OpKind::Sub, y, one);
            uint32_t p = add2(g, OpKind::Pow, x, e);
            uint32_t fa = add2(g, OpKind::Mul, y, p);
            c = add2(g, OpKind::Mul, ct, fa);
            break;
          }
          default: {
            // Ties send the whole gradient to x.
            uint32_t zero = g.scalar(d, 0.0);
            uint32_t m = k == OpKind::Max ? add2(g, OpKind::Ge, x, y) : add2(g, OpKind::Ge, y, x);
            c = g.add(Op::make(OpKind::Where), {m, ct, zero});
          }
        }
        out.emplace_back(x, unbroadcast(g, c, sx));
      }
      if (rel[y]) {
        uint32_t c;
        switch (k) {
          case OpKind::Add: c = ct; break;
          case OpKind::Sub: c = add1(g, OpKind::Neg, ct); break;
          case OpKind::Mul: c = add2(g, OpKind::Mul, ct, x); break;
          case OpKind::Div: {
            uint32_t n = add1(g, OpKind::Neg, ct);
            uint32_t nx = add2(g, OpKind::Mul, n, x);
            uint32_t yy = add2(g, OpKind::Mul, y, y);
            c = add2(g, OpKind::Div, nx, yy);
            break;
          }
          case OpKind::Pow: {
            uint32_t l = add1(g, OpKind::Log, x);
            uint32_t fa = add2(g, OpKind::Mul, me, l);
            c = add2(g, OpKind::Mul, ct, fa);
            break;
          }
          default: {
            uint32_t zero = g.scalar(d, 0.0);
            uint32_t m = k == OpKind::Max ? add2(g, OpKind::Ge, x, y) : add2(g, OpKind::Ge, y, x);
            c = g.add(Op::make(OpKind::Where), {m, zero, ct});
          }
        }
        out.emplace_back(y, unbroadcast(g, c, sy));
      }
      break;
    }
    case OpKind::Where: {
      uint32_t zero = g.scalar(d, 0.0);
      uint32_t c = node.inputs[0], a = node.inputs[1], b = node.inputs[2];
      if (rel[a]) out.emplace_back(a, g.add(Op::make(OpKind::Where), {c, ct, zero}));
      if (rel[b]) out.emplace_back(b, g.add(Op::make(OpKind::Where), {c, zero, ct}));
      break;
    }
    case OpKind::MatMul: {
      // 1-D operands are promoted so one rule covers every rank.
      auto sa = g.shape(x), sb = g.shape(y);
      uint32_t a2 = sa.size() == 1 ? reshape(g, {1, sa[0]}, x) : x;
      uint32_t b2 = sb.size() == 1 ? reshape(g, {sb[0], 1}, y) : y;
      auto cs = g.shape(ct);
      if (sb.size() == 1) cs.push_back(1);
      if (sa.size() == 1) cs.insert(cs.end() - 1, 1);
      uint32_t ct2 = reshape(g, cs, ct);
      if (rel[x]) {
        uint32_t by = swap_last(g, b2);
        uint32_t m = add2(g, OpKind::MatMul, ct2, by);
        auto target = g.shape(a2);
        uint32_t c = unbroadcast(g, m, target);
        out.emplace_back(x, reshape(g, sa, c));
      }
      if (rel[y]) {
        uint32_t c;
        if (sa.size() > 2 && sb.size() == 2) {
          // A shared matrix under a batched operand: flatten the batch (autodiff.rs:445-453).
          size_t k = sb[0], n = sb[1];
          size_t m_total = g.nodes[x].n() / k;
          uint32_t af = reshape(g, {m_total, k}, x);
          uint32_t cf = reshape(g, {m_total, n}, ct2);
          uint32_t ax = swap_last(g, af);
          c = add2(g, OpKind::MatMul, ax, cf);
        } else {
          uint32_t ax = swap_last(g, a2);
          uint32_t m = add2(g, OpKind::MatMul, ax, ct2);
          auto target = g.shape(b2);
          c = unbroadcast(g, m, target);
        }
        out.emplace_back(y, reshape(g, sb, c));
      }
      break;
    }
    case OpKind::Take: {
      Op o = Op::make(OpKind::TakeGrad);
      o.index = node.op.index;
      o.shape = g.shape(x);
      out.emplace_back(x, g.add(std::move(o), {ct, y}));
      break;
    }
    case OpKind::TakeGrad: {
      Op o = Op::make(OpKind::Take);
      o.index = node.op.index;
      out.emplace_back(x, g.add(std::move(o), {ct, y}));
      break;
    }
    case OpKind::TakeAlong: {
      Op o = Op::make(OpKind::TakeAlongGrad);
      o.shape = g.shape(x);
      out.emplace_back(x, g.add(std::move(o), {ct, y}));
      break;
    }
    case OpKind::TakeAlongGrad: out.emplace_back(x, g.add(Op::make(OpKind::TakeAlong), {ct, y})); break;
    case OpKind::Concat: {
      auto shape = node.shape;
      size_t at = 0, axis = node.op.index;
      for (auto input : node.inputs) {
        size_t len = g.shape(input)[axis];
        if (rel[input]) {
          Op s = Op::make(OpKind::Slice);
          s.starts.assign(shape.size(), 0);
          s.stops = shape;
          s.starts[axis] = at;
          s.stops[axis] = at + len;
          out.emplace_back(input, g.add(std::move(s), {ct}));
        }
        at += len;
      }
      break;
    }
    case OpKind::Custom: {
      // Re-instantiate the rule with the real cotangent in place of the placeholder.
      std::map<uint32_t, uint32_t> memo{{node.op.placeholder, ct}};
      uint32_t last = node.op.placeholder;
      for (auto& r : node.op.rules) last = std::max(last, r.second);
      for (uint32_t id = node.op.placeholder + 1; id <= last; ++id) {
        Node n = g.nodes[id];
        bool touches = false;
        for (auto v : n.inputs) touches = touches || memo.count(v);
        if (touches) {
          std::vector<uint32_t> ins;
          for (auto v : n.inputs) ins.push_back(memo.count(v) ? memo[v] : v);
          memo[id] = g.add(n.op, ins);
        }
      }
      for (auto& r : node.op.rules)
        if (rel[r.first]) out.emplace_back(r.first, memo.count(r.second) ? memo[r.second] : r.second);
      break;
    }
    case OpKind::Floor: case OpKind::Argmax: case OpKind::RandUniform: case OpKind::RandNormal:
    case OpKind::KeySplit: case OpKind::Placeholder: case OpKind::ArgTopK: case OpKind::Output:
      break;
    case OpKind::AllReduce: out.emplace_back(x, g.add(Op::make(OpKind::AllReduce), {ct})); break;
    case OpKind::Cumsum: {
      Op o = Op::make(OpKind::Cumsum);
      o.flag_a = !node.op.flag_a;
      out.emplace_back(x, g.add(std::move(o), {ct}));
      break;
    }
    case OpKind::Reduce: {
      auto in_shape = g.shape(x);
      auto keep = in_shape;
      for (size_t a : node.op.shape) keep[a] = 1;
      uint32_t ct_keep = reshape(g, keep, ct);
      uint32_t c;
      if (node.op.reduce == ReduceKind::Sum) {
        Op b = Op::make(OpKind::BroadcastTo);
        b.shape = in_shape;
        c = g.add(std::move(b), {ct_keep});
      } else {
        // Ties share the gradient equally.
        uint32_t mm = reshape(g, keep, me);
        uint32_t mask = node.op.reduce == ReduceKind::Max ? add2(g, OpKind::Ge, x, mm) : add2(g, OpKind::Ge, mm, x);
        uint32_t count = reduce_sum(g, node.op.shape, true, mask);
        uint32_t share = add2(g, OpKind::Div, mask, count);
        c = add2(g, OpKind::Mul, ct_keep, share);
      }
      out.emplace_back(x, c);
      break;
    }
    case OpKind::Reshape: out.emplace_back(x, reshape(g, g.shape(x), ct)); break;
    case OpKind::Transpose: {
      const auto& p = node.op.shape;
      Op o = Op::make(OpKind::Transpose);
      o.shape.assign(p.size(), 0);
      for (size_t k = 0; k < p.size(); ++k) o.shape[p[k]] = k;
      out.emplace_back(x, g.add(std::move(o), {ct}));
      break;
    }
    case OpKind::BroadcastTo: out.emplace_back(x, unbroadcast(g, ct, g.shape(x))); break;
    case OpKind::Slice: {
      Op o = Op::make(OpKind::Pad);
      o.starts = node.op.starts;
      o.shape = g.shape(x);
      out.emplace_back(x, g.add(std::move(o), {ct}));
      break;
    }
    case OpKind::Pad: {
      Op o = Op::make(OpKind::Slice);
      o.starts = node.op.starts;
      const auto& xs = g.shape(x);
      for (size_t k = 0; k < xs.size(); ++k) o.stops.push_back(node.op.starts[k] + xs[k]);
      out.emplace_back(x, g.add(std::move(o), {ct}));
      break;
    }
    case OpKind::Cast: {
      Op o = Op::make(OpKind::Cast);
      o.dtype = g.dtype(x);
      out.emplace_back(x, g.add(std::move(o), {ct}));
      break;
    }
    case OpKind::MatMulT: throw std::logic_error("optimizer output is never differentiated");
    default: throw std::logic_error("rule table reached control flow");
  }
  return out;
}

}  // namespace

std::vector<uint32_t> grad(Graph& g, uint32_t y, const std::vector<uint32_t>& wrts) {
  if (g.nodes[y].n() != 1) {
    Json obs = Json::object();
    obs["output_shape"] = Json(g.shape(y));
    obs["required"] = "single element";
    throw DiagError(diag("GRAD_NON_SCALAR", "error", g.node_json(y), obs, "gradient_of_non_scalar_output", "verified"));
  }
  bool int_wrt = false;
  for (auto w : wrts) int_wrt = int_wrt || g.dtype(w) == DType::I32;
  if (g.dtype(y) == DType::I32 || int_wrt) {
    Json obs = Json::object();
    obs["output_dtype"] = dtype_name(g.dtype(y));
    Json names = Json::array();
    for (auto w : wrts) names.push(dtype_name(g.dtype(w)));
    obs["wrt_dtypes"] = names;
    throw DiagError(diag("GRAD_OF_INTEGER", "error", g.node_json(y), obs, "integers_are_not_differentiable", "verified"));
  }
  size_t end = y;
  auto saved_src = g.cur_source;
  auto saved_origin = g.cur_origin;

  std::vector<bool> rel(end + 1, false);
  for (size_t i = 0; i <= end; ++i) {
    const Node& n = g.nodes[i];
    bool flows = false;
    if (n.op.kind == OpKind::Custom) {
      for (auto& r : n.op.rules) flows = flows || rel[r.first];
    } else if (n.op.is_control_flow()) {
      for (auto x : n.inputs) flows = flows || rel[x];
    } else if (!blocks_gradient(n.op)) {
      for (auto x : n.inputs) flows = flows || rel[x];
    }
    rel[i] = n.dtype != DType::I32 && (std::find(wrts.begin(), wrts.end(), (uint32_t)i) != wrts.end() || flows);
  }

  std::vector<int64_t> cot(end + 1, -1);
  if (rel[end]) cot[end] = g.constant(Tensor::full(g.dtype(y), g.shape(y), 1.0));
  auto accumulate = [&](const Pairs& contributions) {
    for (auto& ic : contributions) {
      uint32_t input = ic.first, c = ic.second;
      if (cot[input] >= 0) cot[input] = add2(g, OpKind::Add, (uint32_t)cot[input], c);
      else cot[input] = c;
    }
  };
  for (size_t i = end + 1; i-- > 0;) {
    if (g.nodes[i].op.is_control_flow()) {
      if (!rel[i]) continue;
      std::map<size_t, uint32_t> cots;
      for (size_t o = i + 1; o <= end; ++o) {
        const Node& n = g.nodes[o];
        if (n.op.kind == OpKind::Output && !n.inputs.empty() && n.inputs[0] == i && cot[o] >= 0) cots[n.op.index] = (uint32_t)cot[o];
      }
      if (cots.empty()) continue;
      g.cur_source = g.nodes[i].source;
      g.cur_origin = (uint32_t)i;
      accumulate(vjp_control(g, i, cots, rel));
      continue;
    }
    if (cot[i] < 0) continue;
    g.cur_source = g.nodes[i].source;
    g.cur_origin = (uint32_t)i;
    accumulate(vjp(g, i, (uint32_t)cot[i], rel));
  }
  g.cur_source = saved_src;
  g.cur_origin = saved_origin;
  std::vector<uint32_t> out;
  for (auto w : wrts) {
    uint32_t id;
    if (w < cot.size() && cot[w] >= 0) {
      id = (uint32_t)cot[w];
    } else {
      Json obs = Json::object();
      obs["output_node"] = y;
      obs["wrt_node"] = w;
      g.notes.push_back(diag("GRAD_DISCONNECTED", "warning", g.node_json(w), obs, "output_does_not_depend_on_input", "verified"));
      id = g.constant(Tensor::full(g.dtype(w), g.shape(w), 0.0));
    }
    g.grads.push_back(GradRecord{y, w, id});
    out.push_back(id);
  }
  return out;
}

}  // namespace rg
