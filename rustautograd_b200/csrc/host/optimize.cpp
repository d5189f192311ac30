// Restates src/optimize.rs (line references below are to that file).
#include "optimize.h"

#include <algorithm>
#include <map>
#include <unordered_map>

#include "plan.h"

namespace rg {

namespace {

constexpr size_t FOLD_LIMIT = 4096;
constexpr size_t CSE_CONST_LIMIT = 16;
constexpr size_t REMAT_MIN = size_t(1) << 14;
constexpr double SEARCH_MIN_GAIN = 0.9;
// egraph.rs:363: iteration and e-node limits of the search (never a time limit).
constexpr size_t SEARCH_ITERATIONS = 6, SEARCH_NODES = 20000;
constexpr size_t COSTLY_REMAT_ABOVE_BYTES = size_t(2) << 30;
// The device's own memory policy (no counterpart in rg): rg rematerialises elementwise values in
// the backward pass to bound the memory of a unified-memory GPU, at the price of recomputing
// them (8 % more algorithmic bytes in a GPT training step). An HBM device keeps the activations
// when the plan without rematerialisation peaks at no more than this; recomputation gives the
// same values, so results do not change.
constexpr size_t DEVICE_KEEP_ACTIVATIONS_BYTES = size_t(48) << 30;
// rg also recomputes transcendental values (exp, tanh...) once the plan would peak above 2 GB;
// the device does so only above this (d512 at batch 512: 1193 instead of 1257 GB of algorithmic
// traffic per step for a 65 instead of 55 GB peak).
constexpr size_t DEVICE_COSTLY_REMAT_ABOVE_BYTES = size_t(96) << 30;

// The value of a constant whose elements are all equal (optimize.rs:45-53).
std::optional<double> splat(const Graph& g, uint32_t id) {
  const Node& n = g.nodes[id];
  if (n.op.kind != OpKind::Const) return std::nullopt;
  const Tensor& t = *n.op.value;
  if (t.n() == 0 || t.n() > FOLD_LIMIT) return std::nullopt;
  double v0 = t.data.get(0);
  for (size_t i = 1; i < t.n(); ++i)
    if (!(t.data.get(i) == v0)) return std::nullopt;
  if (!(v0 == v0)) return std::nullopt;  // NaN never equals itself
  return v0;
}

// optimize.rs:55-77. Never rewrites `x * 0`: that would hide NaN/Inf in `x`.
std::optional<uint32_t> identity(const Graph& g, const Op& op, const std::vector<uint32_t>& ins, const std::vector<size_t>& shape) {
  auto same = [&](uint32_t id) { return g.shape(id) == shape; };
  auto is = [&](uint32_t id, double c) {
    auto s = splat(g, id);
    return s && *s == c;
  };
  switch (op.kind) {
    case OpKind::StopGradient: case OpKind::Custom: return ins[0];
    case OpKind::Add:
      if (is(ins[1], 0.0) && same(ins[0])) return ins[0];
      if (is(ins[0], 0.0) && same(ins[1])) return ins[1];
      return std::nullopt;
    case OpKind::Sub:
      if (is(ins[1], 0.0) && same(ins[0])) return ins[0];
      return std::nullopt;
    case OpKind::Mul:
      if (is(ins[1], 1.0) && same(ins[0])) return ins[0];
      if (is(ins[0], 1.0) && same(ins[1])) return ins[1];
      return std::nullopt;
    case OpKind::Div:
    case OpKind::Pow:
      if (is(ins[1], 1.0) && same(ins[0])) return ins[0];
      return std::nullopt;
    case OpKind::Neg:
      if (g.nodes[ins[0]].op.kind == OpKind::Neg) return g.nodes[ins[0]].inputs[0];
      return std::nullopt;
    case OpKind::Reshape: case OpKind::BroadcastTo:
      if (same(ins[0])) return ins[0];
      return std::nullopt;
    case OpKind::Cast:
      if (op.dtype == g.dtype(ins[0])) return ins[0];
      return std::nullopt;
    case OpKind::Transpose: {
      for (size_t i = 0; i < op.shape.size(); ++i)
        if (op.shape[i] != i) return std::nullopt;
      return ins[0];
    }
    default: return std::nullopt;
  }
}

// optimize.rs:85-93
bool recomputable(const Op& op, bool costly_too) {
  bool elementwise = op.is_unary_elementwise() || op.is_binary_elementwise() || op.kind == OpKind::Where;
  bool costly = op.kind == OpKind::Exp || op.kind == OpKind::Log || op.kind == OpKind::Sin || op.kind == OpKind::Cos ||
                op.kind == OpKind::Tanh || op.kind == OpKind::Sqrt;
  return elementwise && op.kind != OpKind::Pow && (costly_too || !costly);
}

bool is_leaf(const Node& n) { return n.op.kind == OpKind::Input || n.op.kind == OpKind::Const; }

size_t count_kept(const Graph& g, const std::vector<uint32_t>& outputs) {
  auto keep = g.reachable(outputs);
  return (size_t)std::count(keep.begin(), keep.end(), true);
}

// optimize.rs:95-166
std::pair<Graph, std::vector<uint32_t>> rematerialize(const Graph& g, const std::vector<uint32_t>& outputs, const std::vector<bool>& backward,
                                                      size_t min_n, bool costly_too, OptStats& st) {
  auto keep = g.reachable(outputs);
  size_t N = g.nodes.size();
  auto large = [&](uint32_t id) { return g.nodes[id].n() >= min_n; };
  std::vector<bool> retained(N, false);
  for (size_t i = 0; i < N; ++i)
    if (keep[i] && backward[i])
      for (auto x : g.nodes[i].inputs) retained[x] = retained[x] || !backward[x];
  std::vector<bool> remat(N, false);
  for (size_t i = N; i-- > 0;) {
    const Node& n = g.nodes[i];
    if (!retained[i] || backward[i] || !recomputable(n.op, costly_too) || !large((uint32_t)i)) continue;
    std::vector<uint32_t> fresh;
    for (auto x : n.inputs)
      if (large(x) && !retained[x] && !is_leaf(g.nodes[x])) fresh.push_back(x);
    fresh.erase(std::unique(fresh.begin(), fresh.end()), fresh.end());  // Vec::dedup
    if (fresh.size() <= 1) {
      remat[i] = true;
      retained[i] = false;
      for (auto x : n.inputs) retained[x] = true;
    }
  }
  Graph h;
  std::vector<uint32_t> map(N, UINT32_MAX);
  std::vector<int64_t> clone(N, -1);
  std::function<uint32_t(uint32_t)> value = [&](uint32_t i) -> uint32_t {
    if (!remat[i]) return map[i];
    if (clone[i] >= 0) return (uint32_t)clone[i];
    const Node& n = g.nodes[i];
    std::vector<uint32_t> ins;
    for (auto x : n.inputs) ins.push_back(value(x));
    h.cur_source = n.source;
    uint32_t id = h.add(n.op, ins);
    clone[i] = id;
    st.rematerialized += 1;
    return id;
  };
  for (size_t i = 0; i < N; ++i) {
    const Node& n = g.nodes[i];
    if (n.op.kind == OpKind::Input) {
      h.cur_source = n.source;
      map[i] = h.input(n.shape, n.dtype);
      h.nodes[map[i]].op = n.op;
      continue;
    }
    if (!keep[i]) continue;
    std::vector<uint32_t> ins;
    for (auto x : n.inputs) ins.push_back(backward[i] ? value(x) : map[x]);
    h.cur_source = n.source;
    map[i] = n.op.kind == OpKind::Const ? h.constant(n.op.value) : h.add(n.op, ins);
  }
  std::vector<uint32_t> out;
  for (auto o : outputs) out.push_back(map[o]);
  return {std::move(h), std::move(out)};
}

// The device's own rewrite (no counterpart in rg): a sum of zero-padded blocks that tile one axis
// of their common shape, as the gradient of slices taken along that axis comes out of autodiff
// (the q, k, v split of an attention layer: pad each gradient to the full tensor, then add), is
// the concatenation of the blocks. The sum writes every padded tensor in full and reads them all
// again; the concatenation reads each block once. Every element equals the sum's (x + 0 = x),
// except that a block's -0 stays -0 where the sum gives +0.
// Collects the blocks of the sum rooted at `id`: (start on the padded axis, block id).
bool pad_blocks(const Graph& g, uint32_t id, const std::vector<size_t>& shape, DType dt, int* axis,
                std::vector<std::pair<size_t, uint32_t>>* blocks, int depth) {
  const Node& n = g.nodes[id];
  if (n.shape != shape || n.dtype != dt || depth > 64) return false;
  if (n.op.kind == OpKind::Add)
    return n.inputs.size() == 2 && pad_blocks(g, n.inputs[0], shape, dt, axis, blocks, depth + 1) &&
           pad_blocks(g, n.inputs[1], shape, dt, axis, blocks, depth + 1);
  if (n.op.kind != OpKind::Pad || n.inputs.size() != 1) return false;
  const auto& xs = g.shape(n.inputs[0]);
  if (xs.size() != shape.size() || n.op.starts.size() != shape.size()) return false;
  int a = -1;
  for (size_t d = 0; d < shape.size(); ++d) {
    if (xs[d] == shape[d] && n.op.starts[d] == 0) continue;
    if (a >= 0) return false;  // padded along two axes
    a = (int)d;
  }
  if (a < 0 || (*axis >= 0 && *axis != a)) return false;
  *axis = a;
  blocks->emplace_back(n.op.starts[a], n.inputs[0]);
  return true;
}

// The concatenation equal to the sum `a + b`, when the blocks tile the padded axis exactly.
std::optional<std::pair<Op, std::vector<uint32_t>>> padded_sum_as_concat(const Graph& g, uint32_t a, uint32_t b, const std::vector<size_t>& shape,
                                                                         DType dt) {
  int axis = -1;
  std::vector<std::pair<size_t, uint32_t>> blocks;
  if (!pad_blocks(g, a, shape, dt, &axis, &blocks, 0) || !pad_blocks(g, b, shape, dt, &axis, &blocks, 0)) return std::nullopt;
  std::sort(blocks.begin(), blocks.end());
  size_t pos = 0;
  std::vector<uint32_t> ins;
  for (auto& [start, id] : blocks) {
    if (start != pos) return std::nullopt;  // a gap or an overlap
    pos += g.shape(id)[(size_t)axis];
    ins.push_back(id);
  }
  if (pos != shape[(size_t)axis]) return std::nullopt;
  Op op = Op::make(OpKind::Concat);
  op.index = (size_t)axis;
  return std::make_pair(op, ins);
}

struct Simplified {
  Graph g;
  std::vector<uint32_t> out;
  OptStats st;
  std::vector<bool> backward;
};

// optimize.rs:286-403. Single forward rewrite: SSA order lets folds and identities cascade.
// `concat_pads` adds the device's padded-sum rewrite (above).
Simplified simplify(const Graph& g, const std::vector<uint32_t>& outputs, bool flip_transposes, bool concat_pads = false) {
  auto keep = g.reachable(outputs);
  Simplified r;
  r.st.nodes_before = (size_t)std::count(keep.begin(), keep.end(), true);
  Graph& ng = r.g;
  std::vector<uint32_t> map(g.nodes.size(), UINT32_MAX);
  std::unordered_map<std::string, uint32_t> seen;
  std::vector<bool>& backward = r.backward;

  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& node = g.nodes[i];
    ng.cur_source = node.source;
    ng.cur_origin.reset();
    if (node.op.kind == OpKind::Input) {
      map[i] = ng.input(node.shape, node.dtype);
      ng.nodes[map[i]].op = node.op;  // reverse scans renumber their inputs
      backward.resize(ng.nodes.size(), false);
      continue;
    }
    if (!keep[i]) continue;
    std::vector<uint32_t> ins;
    for (auto x : node.inputs) ins.push_back(map[x]);

    if (auto existing = identity(ng, node.op, ins, node.shape)) {
      map[i] = *existing;
      r.st.simplified += 1;
      continue;
    }
    Op op = node.op;
    if (concat_pads && op.kind == OpKind::Add && ins.size() == 2) {
      if (auto c = padded_sum_as_concat(ng, ins[0], ins[1], node.shape, node.dtype)) {
        op = c->first;
        ins = c->second;
        r.st.simplified += 1;
      }
    }
    if (op.kind == OpKind::Pow) {
      auto s = splat(ng, ins[1]);
      if (s && *s == 2.0 && ng.shape(ins[0]) == node.shape) {
        op = Op::make(OpKind::Mul);
        ins = {ins[0], ins[0]};
        r.st.simplified += 1;
      }
    }
    // Binary kernels broadcast by themselves, so a materialised broadcast is a wasted copy.
    if (op.is_binary_elementwise()) {
      for (int k = 0; k < 2; ++k) {
        const Node& n = ng.nodes[ins[k]];
        if (n.op.kind == OpKind::BroadcastTo) {
          uint32_t source = n.inputs[0];
          uint32_t other = ins[1 - k];
          std::vector<size_t> joint;
          if (broadcast_shapes(ng.shape(source), ng.shape(other), &joint) && joint == node.shape) {
            ins[k] = source;
            r.st.simplified += 1;
          }
        }
      }
    }
    // A transposed operand is read through a flag; the copy then goes away with DCE.
    if (flip_transposes && op.kind == OpKind::MatMul) {
      auto flipped = [&](uint32_t id) -> std::optional<uint32_t> {
        const Node& n = ng.nodes[id];
        if (n.op.kind != OpKind::Transpose) return std::nullopt;
        const auto& p = n.op.shape;
        if (p.size() < 2) return std::nullopt;
        for (size_t a = 0; a < p.size(); ++a) {
          bool ok = a + 2 < p.size() ? a == p[a] : a + p[a] == 2 * p.size() - 3;
          if (!ok) return std::nullopt;
        }
        return n.inputs[0];
      };
      auto fa = flipped(ins[0]);
      auto fb = flipped(ins[1]);
      if (fa || fb) {
        op = Op::make(OpKind::MatMulT);
        op.flag_a = (bool)fa;
        op.flag_b = (bool)fb;
        ins = {fa ? *fa : ins[0], fb ? *fb : ins[1]};
        r.st.simplified += 1;
      }
    }
    bool foldable = !op.is_control_flow() && op.kind != OpKind::Output && op.kind != OpKind::AllReduce && !ins.empty() && node.n() <= FOLD_LIMIT;
    for (auto x : ins) foldable = foldable && ng.nodes[x].op.kind == OpKind::Const;
    if (foldable) {
      Graph tmp;
      std::vector<uint32_t> ids;
      for (auto x : ins) ids.push_back(tmp.constant(ng.nodes[x].op.value));
      uint32_t id = tmp.add(op, ids);
      auto value = eval(tmp, {id}, {});
      Op c = Op::make(OpKind::Const);
      c.value = std::make_shared<const Tensor>(std::move(value[0]));
      op = std::move(c);
      ins.clear();
      r.st.folded += 1;
    }
    bool big_const = op.kind == OpKind::Const && op.value->n() > CSE_CONST_LIMIT;
    std::string key;
    if (!big_const) {
      key = op.key();
      key += '|';
      for (auto x : ins) key += std::to_string(x) + ",";
      auto it = seen.find(key);
      if (it != seen.end()) {
        map[i] = it->second;
        r.st.cse += 1;
        continue;
      }
    }
    uint32_t id = op.kind == OpKind::Const ? ng.constant(op.value) : ng.add(op, ins);
    ng.nodes[id].origin = node.origin;  // only presence is read after this point
    backward.resize(ng.nodes.size(), false);
    backward[id] = node.origin.has_value();
    if (!big_const) seen[key] = id;
    map[i] = id;
  }
  for (auto o : outputs) r.out.push_back(map[o]);
  backward.resize(ng.nodes.size(), false);
  return r;
}

// `gpu`: planning for the device, whose plans keep every activation (no rematerialisation) while
// that plan's peak live bytes stay within DEVICE_KEEP_ACTIVATIONS_BYTES; above it rg's policy,
// escalating to transcendental values only above DEVICE_COSTLY_REMAT_ABOVE_BYTES.
OptResult finish(const Graph& ng, const std::vector<uint32_t>& out, const std::vector<bool>& backward, OptStats st, bool gpu = false) {
  if (gpu && Plan::build(ng, out, true).peak_live_bytes <= DEVICE_KEEP_ACTIVATIONS_BYTES) {
    st.nodes_after = count_kept(ng, out);
    return OptResult{ng, out, st};
  }
  auto hr = rematerialize(ng, out, backward, REMAT_MIN, false, st);
  if (Plan::build(hr.first, hr.second, true).peak_live_bytes > (gpu ? DEVICE_COSTLY_REMAT_ABOVE_BYTES : COSTLY_REMAT_ABOVE_BYTES)) {
    st.rematerialized = 0;
    hr = rematerialize(ng, out, backward, REMAT_MIN, true, st);
  }
  st.nodes_after = count_kept(hr.first, hr.second);
  return OptResult{std::move(hr.first), std::move(hr.second), st};
}

}  // namespace

bool parse_opt_mode(const std::string& s, OptMode* m) {
  if (s == "none") *m = OptMode::None;
  else if (s == "standard") *m = OptMode::Standard;
  else if (s == "search-exact") *m = OptMode::SearchExact;
  else if (s == "search-linear") *m = OptMode::SearchLinear;
  else if (s == "search") *m = OptMode::Search;
  else if (s == "auto") *m = OptMode::Auto;
  else return false;
  return true;
}

Json OptStats::json() const {
  Json j = Json::object();
  j["nodes_before"] = nodes_before;
  j["nodes_after"] = nodes_after;
  j["constants_folded"] = folded;
  j["algebraic_simplified"] = simplified;
  j["cse_merged"] = cse;
  j["rematerialized"] = rematerialized;
  if (search) {
    Json s = Json::object();
    s["accepted"] = search->accepted;
    s["iterations"] = search->iterations;
    s["egraph_nodes"] = search->egraph_nodes;
    s["cost_before"] = search->cost_before;
    s["cost_after"] = search->cost_after;
    j["search"] = s;
  } else {
    j["search"] = nullptr;
  }
  return j;
}

OptResult optimize(const Graph& g, const std::vector<uint32_t>& outputs) { return optimize_mode(g, outputs, OptMode::Standard); }

// optimize.rs:210-246
OptResult optimize_mode(const Graph& g, const std::vector<uint32_t>& outputs, OptMode mode, bool gpu) {
  if (mode == OptMode::Auto) mode = OptMode::Standard;  // compile() resolves Auto before this point
  if (mode == OptMode::None) {
    size_t k = count_kept(g, outputs);
    OptStats st;
    st.nodes_before = st.nodes_after = k;
    return OptResult{g, outputs, st};
  }
  if (mode == OptMode::Standard) {
    Simplified s = simplify(g, outputs, true, gpu);
    return finish(s.g, s.out, s.backward, s.st, gpu);
  }
  Simplified baseline = simplify(g, outputs, true, gpu);
  Simplified first = simplify(g, outputs, false);
  size_t before = count_kept(g, outputs);
  if (mode == OptMode::SearchLinear && !has_matrix_structure(first.g, first.out)) {
    baseline.st.nodes_before = before;
    return finish(baseline.g, baseline.out, baseline.backward, baseline.st, gpu);
  }
  SearchStats ss;
  std::optional<Simplified> candidate;
  const CostModel& model = gpu ? CostModel::CUDA : CostModel::CPU;
  const int set = mode == OptMode::Search ? 2 : mode == OptMode::SearchLinear ? 1 : 0;
  if (auto found = search(first.g, first.out, model, set, SEARCH_ITERATIONS, SEARCH_NODES, &ss)) candidate = simplify(found->first, found->second, true, gpu);
  // Compare final forms: both sides have folded constants and flagged transposes.
  ss.cost_before = model.graph_cost(baseline.g, baseline.out);
  ss.cost_after = candidate ? model.graph_cost(candidate->g, candidate->out) : ss.cost_before;
  ss.accepted = candidate.has_value() && ss.cost_after < ss.cost_before * SEARCH_MIN_GAIN;
  Simplified& chosen = ss.accepted ? *candidate : baseline;
  chosen.st.nodes_before = before;
  chosen.st.search = ss;
  return finish(chosen.g, chosen.out, chosen.backward, chosen.st, gpu);
}

// optimize.rs:260-277
bool has_matrix_structure(const Graph& g, const std::vector<uint32_t>& outputs) {
  auto keep = g.reachable(outputs);
  auto is_product = [&](uint32_t id) {
    const Node* n = &g.nodes[id];
    if (n->op.kind == OpKind::Transpose && n->op.shape == std::vector<size_t>{1, 0}) n = &g.nodes[n->inputs[0]];
    return n->op.kind == OpKind::MatMul;
  };
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!keep[i]) continue;
    const Node& n = g.nodes[i];
    if (n.op.kind == OpKind::MatMul) {
      for (auto x : n.inputs)
        if (is_product(x)) return true;
    } else if (n.op.kind == OpKind::Add) {
      bool all = true;
      for (auto x : n.inputs) all = all && is_product(x);
      if (all) return true;
    }
  }
  return false;
}

}  // namespace rg
