// Equality saturation over the graph's arithmetic (restates the behaviour of src/egraph.rs).
//
// rg runs the `egg` crate (0.11.0, Cargo.lock) with three rule sets and picks the cheapest form
// of every equivalence class under a per-node cost model. This file is an e-graph of its own in
// the same published scheme (Willsey et al., "egg: Fast and extensible equality saturation",
// POPL 2021): hash-consed e-nodes over union-find e-classes, rule matches collected on a fixed
// e-graph and then applied, congruence restored by deferred rebuilding, a back-off scheduler for
// rules that match too often, node and iteration limits (never time, so a program always gets
// the same plan), and tree-cost extraction. The rules and the cost models are rg's
// (egraph.rs:126-233); a rule applies only when its result has exactly the matched class's
// shape and dtype (egraph.rs:94-124). Only `search-*` optimisation modes call it.
#include <algorithm>
#include <cmath>
#include <functional>
#include <limits>
#include <map>
#include <memory>
#include <unordered_map>

#include "optimize.h"

namespace rg {

namespace {

// ---- symbols ----
enum class Sym : uint8_t { Leaf, Opaque, Add, Sub, Mul, Div, Neg, Where, MatMul, T, MMTA, MMTB, MMTT };

struct ENode {
  Sym sym = Sym::Leaf;
  uint32_t key = 0;  // Leaf / Opaque: index into the leaf / opaque tables
  std::vector<uint32_t> kids;
  bool operator==(const ENode& o) const { return sym == o.sym && key == o.key && kids == o.kids; }
};

struct ENodeHash {
  size_t operator()(const ENode& n) const {
    size_t h = (size_t)n.sym * 1000003u ^ (size_t)n.key * 7919u;
    for (auto k : n.kids) h = h * 31 + k + 0x9e3779b9;
    return h;
  }
};

struct Info {
  std::vector<size_t> shape;
  DType dtype = DType::F32;
  std::optional<double> splat;  // every element equals this constant
  bool valid = false;
};

Op op_of_sym(Sym s) {
  switch (s) {
    case Sym::Add: return Op::make(OpKind::Add);
    case Sym::Sub: return Op::make(OpKind::Sub);
    case Sym::Mul: return Op::make(OpKind::Mul);
    case Sym::Div: return Op::make(OpKind::Div);
    case Sym::Neg: return Op::make(OpKind::Neg);
    case Sym::Where: return Op::make(OpKind::Where);
    case Sym::MatMul: return Op::make(OpKind::MatMul);
    case Sym::T: {
      Op o = Op::make(OpKind::Transpose);
      o.shape = {1, 0};
      return o;
    }
    default: {
      Op o = Op::make(OpKind::MatMulT);
      o.flag_a = s == Sym::MMTA || s == Sym::MMTT;
      o.flag_b = s == Sym::MMTB || s == Sym::MMTT;
      return o;
    }
  }
}

// Shape and dtype of a rule-built node from its children (egraph.rs:64-92).
Info derive(Sym s, const std::vector<const Info*>& kids) {
  Info bad;
  for (auto* k : kids)
    if (!k->valid) return bad;
  if ((s == Sym::Add || s == Sym::Sub || s == Sym::Mul || s == Sym::Div) && kids.size() == 2) {
    if (kids[0]->dtype != kids[1]->dtype) return bad;
    Info r;
    if (!broadcast_shapes(kids[0]->shape, kids[1]->shape, &r.shape)) return bad;
    r.dtype = kids[0]->dtype;
    r.valid = true;
    return r;
  }
  if (s == Sym::Neg && kids.size() == 1) {
    Info r = *kids[0];
    r.splat.reset();
    return r;
  }
  // Everything else: the graph's own inference on a probe graph.
  Graph probe;
  std::vector<uint32_t> ids;
  for (auto* k : kids) ids.push_back(probe.input(k->shape, k->dtype));
  try {
    uint32_t id = probe.add(op_of_sym(s), ids);
    Info r;
    r.shape = probe.shape(id);
    r.dtype = probe.dtype(id);
    r.valid = true;
    return r;
  } catch (...) {
    return bad;
  }
}

// ---- the e-graph ----
struct EClass {
  std::vector<ENode> nodes;
  std::vector<std::pair<ENode, uint32_t>> parents;  // (parent node, its class) using this class
  Info data;
};

class EGraph {
 public:
  std::vector<uint32_t> uf;
  std::vector<EClass> cls;
  std::unordered_map<ENode, uint32_t, ENodeHash> memo;
  std::vector<uint32_t> dirty;
  size_t n_nodes = 0;

  uint32_t find(uint32_t a) const {
    while (uf[a] != a) a = uf[a];
    return a;
  }
  uint32_t find_compress(uint32_t a) {
    uint32_t r = find(a);
    while (uf[a] != r) {
      uint32_t n = uf[a];
      uf[a] = r;
      a = n;
    }
    return r;
  }
  ENode canon(ENode n) const {
    for (auto& k : n.kids) k = find(k);
    return n;
  }
  // Adds a node (with the Info it carries when it is a leaf or opaque source node).
  uint32_t add(ENode n, const Info* given = nullptr) {
    n = canon(n);
    auto it = memo.find(n);
    if (it != memo.end()) return find(it->second);
    uint32_t id = (uint32_t)cls.size();
    uf.push_back(id);
    cls.emplace_back();
    if (given) {
      cls[id].data = *given;
    } else {
      std::vector<const Info*> ki;
      for (auto k : n.kids) ki.push_back(&cls[k].data);
      cls[id].data = derive(n.sym, ki);
    }
    cls[id].nodes.push_back(n);
    for (auto k : n.kids) cls[k].parents.push_back({n, id});
    memo[n] = id;
    ++n_nodes;
    return id;
  }
  bool merge(uint32_t a, uint32_t b) {
    a = find_compress(a);
    b = find_compress(b);
    if (a == b) return false;
    if (cls[a].nodes.size() + cls[a].parents.size() < cls[b].nodes.size() + cls[b].parents.size()) std::swap(a, b);
    uf[b] = a;
    auto& A = cls[a];
    auto& B = cls[b];
    A.nodes.insert(A.nodes.end(), B.nodes.begin(), B.nodes.end());
    A.parents.insert(A.parents.end(), B.parents.begin(), B.parents.end());
    if (!A.data.splat && B.data.splat) A.data.splat = B.data.splat;
    B.nodes.clear();
    B.parents.clear();
    dirty.push_back(a);
    return true;
  }
  // Restores the hash-cons and congruence after merges (deferred rebuilding).
  void rebuild() {
    while (!dirty.empty()) {
      std::vector<uint32_t> todo;
      todo.swap(dirty);
      for (uint32_t c : todo) {
        c = find_compress(c);
        auto parents = std::move(cls[c].parents);
        cls[c].parents.clear();
        for (auto& [pn, pc] : parents) memo.erase(pn);
        std::unordered_map<ENode, uint32_t, ENodeHash> seen;
        for (auto& [pn, pc] : parents) {
          ENode n = canon(pn);
          uint32_t owner = find(pc);
          auto it = seen.find(n);
          if (it != seen.end()) {
            merge(it->second, owner);
            owner = find(owner);
          }
          seen[n] = owner;
          auto m = memo.find(n);
          if (m != memo.end() && find(m->second) != owner) merge(m->second, owner);
          memo[n] = find(owner);
        }
        c = find(c);
        for (auto& [n, o] : seen) cls[c].parents.push_back({n, find(o)});
      }
    }
    // Canonical, duplicate-free node lists.
    for (uint32_t c = 0; c < cls.size(); ++c) {
      if (find(c) != c) continue;
      auto& v = cls[c].nodes;
      for (auto& n : v) n = canon(n);
      std::vector<ENode> u;
      for (auto& n : v)
        if (std::find(u.begin(), u.end(), n) == u.end()) u.push_back(n);
      v.swap(u);
    }
  }
};

// ---- rules: s-expression patterns over the symbols above ----
struct Pat {
  bool var = false;
  int v = -1;  // variable number
  Sym sym = Sym::Leaf;
  std::vector<Pat> kids;
};

Sym sym_of_name(const std::string& s) {
  static const std::map<std::string, Sym> m = {{"add", Sym::Add}, {"sub", Sym::Sub},   {"mul", Sym::Mul},     {"div", Sym::Div},
                                               {"neg", Sym::Neg}, {"where", Sym::Where}, {"matmul", Sym::MatMul}, {"t", Sym::T},
                                               {"mm-ta", Sym::MMTA}, {"mm-tb", Sym::MMTB}, {"mm-tt", Sym::MMTT}};
  return m.at(s);
}

Pat parse(const std::string& s, size_t& i, std::map<std::string, int>& vars) {
  while (s[i] == ' ') ++i;
  Pat p;
  if (s[i] == '?') {
    size_t j = i;
    while (j < s.size() && s[j] != ' ' && s[j] != ')') ++j;
    std::string name = s.substr(i, j - i);
    i = j;
    p.var = true;
    auto it = vars.find(name);
    p.v = it != vars.end() ? it->second : (vars[name] = (int)vars.size());
    return p;
  }
  ++i;  // '('
  size_t j = i;
  while (s[j] != ' ' && s[j] != ')') ++j;
  p.sym = sym_of_name(s.substr(i, j - i));
  i = j;
  while (true) {
    while (s[i] == ' ') ++i;
    if (s[i] == ')') {
      ++i;
      break;
    }
    p.kids.push_back(parse(s, i, vars));
  }
  return p;
}

struct Rule {
  std::string name;
  Pat lhs, rhs;
  int nvars = 0;
};

Rule rule(const std::string& name, const std::string& l, const std::string& r) {
  Rule x;
  x.name = name;
  std::map<std::string, int> vars;
  size_t i = 0;
  x.lhs = parse(l, i, vars);
  i = 0;
  x.rhs = parse(r, i, vars);
  x.nvars = (int)vars.size();
  return x;
}

// egraph.rs:126-168
std::vector<Rule> rules_for(int set) {  // 0 exact, 1 linear, 2 rounding
  std::vector<Rule> r = {
      rule("add-comm", "(add ?a ?b)", "(add ?b ?a)"),
      rule("mul-comm", "(mul ?a ?b)", "(mul ?b ?a)"),
      rule("neg-neg", "(neg (neg ?a))", "?a"),
      rule("sub-to-add", "(sub ?a ?b)", "(add ?a (neg ?b))"),
      rule("add-to-sub", "(add ?a (neg ?b))", "(sub ?a ?b)"),
      rule("neg-mul", "(mul (neg ?a) ?b)", "(neg (mul ?a ?b))"),
      rule("mul-neg", "(neg (mul ?a ?b))", "(mul (neg ?a) ?b)"),
      rule("neg-div", "(div (neg ?a) ?b)", "(neg (div ?a ?b))"),
      rule("t-t", "(t (t ?a))", "?a"),
      rule("mm-ta", "(matmul (t ?a) ?b)", "(mm-ta ?a ?b)"),
      rule("mm-tb", "(matmul ?a (t ?b))", "(mm-tb ?a ?b)"),
      rule("mm-tt", "(mm-ta ?a (t ?b))", "(mm-tt ?a ?b)"),
      rule("mm-tt2", "(mm-tb (t ?a) ?b)", "(mm-tt ?a ?b)"),
      rule("where-same", "(where ?c ?a ?a)", "?a"),
  };
  if (set >= 1) {
    r.push_back(rule("matmul-assoc", "(matmul (matmul ?a ?b) ?c)", "(matmul ?a (matmul ?b ?c))"));
    r.push_back(rule("matmul-assoc-r", "(matmul ?a (matmul ?b ?c))", "(matmul (matmul ?a ?b) ?c)"));
    r.push_back(rule("matmul-factor-l", "(add (matmul ?a ?x) (matmul ?a ?y))", "(matmul ?a (add ?x ?y))"));
    r.push_back(rule("matmul-factor-r", "(add (matmul ?x ?a) (matmul ?y ?a))", "(matmul (add ?x ?y) ?a)"));
    r.push_back(rule("t-matmul", "(t (matmul ?a ?b))", "(matmul (t ?b) (t ?a))"));
    r.push_back(rule("matmul-t", "(matmul (t ?b) (t ?a))", "(t (matmul ?a ?b))"));
  }
  if (set >= 2) {
    r.push_back(rule("add-assoc", "(add (add ?a ?b) ?c)", "(add ?a (add ?b ?c))"));
    r.push_back(rule("add-assoc-r", "(add ?a (add ?b ?c))", "(add (add ?a ?b) ?c)"));
    r.push_back(rule("mul-assoc", "(mul (mul ?a ?b) ?c)", "(mul ?a (mul ?b ?c))"));
    r.push_back(rule("mul-assoc-r", "(mul ?a (mul ?b ?c))", "(mul (mul ?a ?b) ?c)"));
    r.push_back(rule("factor", "(add (mul ?a ?x) (mul ?a ?y))", "(mul ?a (add ?x ?y))"));
    r.push_back(rule("distribute", "(mul ?a (add ?x ?y))", "(add (mul ?a ?x) (mul ?a ?y))"));
    r.push_back(rule("div-div", "(div (div ?x ?y) ?z)", "(div ?x (mul ?y ?z))"));
    r.push_back(rule("mul-div", "(div (mul ?x ?y) ?z)", "(mul ?x (div ?y ?z))"));
  }
  return r;
}

using Subst = std::vector<int64_t>;  // variable -> class, -1 unbound

void match(const EGraph& eg, const Pat& p, uint32_t c, Subst s, std::vector<Subst>& out) {
  c = eg.find(c);
  if (p.var) {
    if (s[p.v] < 0) {
      s[p.v] = c;
      out.push_back(std::move(s));
    } else if (eg.find((uint32_t)s[p.v]) == c) {
      out.push_back(std::move(s));
    }
    return;
  }
  for (const ENode& n : eg.cls[c].nodes) {
    if (n.sym != p.sym || n.kids.size() != p.kids.size()) continue;
    std::vector<Subst> cur = {s};
    for (size_t k = 0; k < p.kids.size() && !cur.empty(); ++k) {
      std::vector<Subst> next;
      for (auto& cs : cur) match(eg, p.kids[k], n.kids[k], cs, next);
      cur.swap(next);
    }
    for (auto& cs : cur) out.push_back(std::move(cs));
  }
}

// Info of every node of an instantiated pattern, without adding it; the result's Info last.
Info rhs_info(const EGraph& eg, const Pat& p, const Subst& s) {
  if (p.var) return eg.cls[eg.find((uint32_t)s[p.v])].data;
  std::vector<Info> kids;
  for (auto& k : p.kids) kids.push_back(rhs_info(eg, k, s));
  std::vector<const Info*> ptr;
  for (auto& k : kids) ptr.push_back(&k);
  return derive(p.sym, ptr);
}

uint32_t instantiate(EGraph& eg, const Pat& p, const Subst& s) {
  if (p.var) return eg.find((uint32_t)s[p.v]);
  ENode n;
  n.sym = p.sym;
  for (auto& k : p.kids) n.kids.push_back(instantiate(eg, k, s));
  return eg.add(std::move(n));
}

}  // namespace

// ---- cost models (egraph.rs:170-233) ----
const CostModel CostModel::CPU = {200.0, 0.06, 0.0015, 0.6, 1.4};
const CostModel CostModel::METAL = {30000.0, 0.1, 0.004, 0.05, 0.15};
// B200 (CUDA graph launches, 3xTF32 GEMMs near 170 TFLOP/s, HBM near 6 TB/s): a launch costs a
// few microseconds, a multiplication far more than an element written.
const CostModel CostModel::CUDA = {3000.0, 0.0007, 0.012, 0.0003, 0.0015};

double CostModel::node(const Op& op, const std::vector<size_t>& shape, const std::vector<const std::vector<size_t>*>& args) const {
  const double n = (double)product(shape);
  const double base = per_op + per_element * n;
  switch (op.kind) {
    case OpKind::Input: case OpKind::Const: case OpKind::Reshape: case OpKind::StopGradient: case OpKind::Output: case OpKind::Custom:
      return 0.0;
    case OpKind::MatMul: {
      double k = args[0]->empty() ? 1.0 : (double)args[0]->back();
      return base + per_flop * n * k;
    }
    case OpKind::MatMulT: {
      const auto& a = *args[0];
      double k = a.size() >= 2 ? (double)(op.flag_a ? a[a.size() - 2] : a.back()) : (a.empty() ? 1.0 : (double)a[0]);
      return base + per_flop * n * k;
    }
    case OpKind::Transpose: return per_op + per_transpose_element * n;
    case OpKind::Exp: case OpKind::Log: case OpKind::Sin: case OpKind::Cos: case OpKind::Tanh: return base + per_math_element * n;
    case OpKind::Pow: return base + 16.0 * per_math_element * n;
    case OpKind::Div: case OpKind::Sqrt: return base + 0.2 * per_math_element * n;
    default: return base;
  }
}

double CostModel::graph_cost(const Graph& g, const std::vector<uint32_t>& outputs) const {
  auto keep = g.reachable(outputs);
  double total = 0;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!keep[i]) continue;
    const Node& n = g.nodes[i];
    bool constant = !n.inputs.empty();
    for (auto x : n.inputs) constant = constant && g.nodes[x].op.kind == OpKind::Const;
    if (constant) continue;
    std::vector<const std::vector<size_t>*> args;
    for (auto x : n.inputs) args.push_back(&g.nodes[x].shape);
    total += node(n.op, n.shape, args);
  }
  return total;
}

// egraph.rs:367-427
std::optional<std::pair<Graph, std::vector<uint32_t>>> search(const Graph& g, const std::vector<uint32_t>& outputs, const CostModel& model,
                                                              int rule_set, size_t iter_limit, size_t node_limit, SearchStats* st) {
  auto keep = g.reachable(outputs);
  EGraph eg;
  std::vector<uint32_t> cls_of(g.nodes.size(), 0);
  std::vector<Op> opaque_ops;
  std::map<std::string, uint32_t> opaque_key;
  std::vector<uint32_t> leaf_node;  // Leaf key -> source node
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    const bool input = n.op.kind == OpKind::Input;
    if (!keep[i] && !input) continue;
    ENode e;
    Info info;
    info.shape = n.shape;
    info.dtype = n.dtype;
    info.valid = true;
    const Info* given = nullptr;
    if (input || n.op.kind == OpKind::Const) {
      e.sym = Sym::Leaf;
      e.key = (uint32_t)leaf_node.size();
      leaf_node.push_back((uint32_t)i);
      if (n.op.kind == OpKind::Const && n.op.value && n.op.value->n() <= 4096) {
        auto v = n.op.value->data.to_f64();
        if (!v.empty() && std::all_of(v.begin(), v.end(), [&](double x) { return x == v[0]; })) info.splat = v[0];
      }
      given = &info;
    } else {
      switch (n.op.kind) {
        case OpKind::Add: e.sym = Sym::Add; break;
        case OpKind::Sub: e.sym = Sym::Sub; break;
        case OpKind::Mul: e.sym = Sym::Mul; break;
        case OpKind::Div: e.sym = Sym::Div; break;
        case OpKind::Neg: e.sym = Sym::Neg; break;
        case OpKind::Where: e.sym = Sym::Where; break;
        case OpKind::MatMul: e.sym = Sym::MatMul; break;
        default:
          if (n.op.kind == OpKind::Transpose && n.op.shape == std::vector<size_t>{1, 0}) {
            e.sym = Sym::T;
          } else {
            // Opaque to the rules; equal ops (attributes included) share a symbol, control
            // flow by identity.
            e.sym = Sym::Opaque;
            std::string k = n.op.is_control_flow() ? "cf" + std::to_string(i) : n.op.key() + "|" + std::to_string((int)n.dtype);
            auto it = opaque_key.find(k);
            if (it == opaque_key.end()) {
              it = opaque_key.emplace(k, (uint32_t)opaque_ops.size()).first;
              opaque_ops.push_back(n.op);
            }
            e.key = it->second;
            given = &info;
          }
      }
      for (auto x : n.inputs) e.kids.push_back(cls_of[x]);
    }
    cls_of[i] = eg.add(e, given);
  }

  // Saturation with a back-off scheduler: a rule matching more than its threshold is skipped
  // for a while, with threshold and ban length doubling each time.
  auto rules = rules_for(rule_set);
  std::vector<size_t> banned_until(rules.size(), 0), times_banned(rules.size(), 0);
  const size_t match_limit = 1000, ban_length = 5;
  size_t it = 0;
  for (; it < iter_limit; ++it) {
    std::vector<std::pair<size_t, std::vector<std::pair<uint32_t, Subst>>>> found;
    for (size_t r = 0; r < rules.size(); ++r) {
      if (banned_until[r] > it) continue;
      std::vector<std::pair<uint32_t, Subst>> ms;
      for (uint32_t c = 0; c < eg.cls.size(); ++c) {
        if (eg.find(c) != c) continue;
        std::vector<Subst> out;
        match(eg, rules[r].lhs, c, Subst(rules[r].nvars, -1), out);
        for (auto& s : out) ms.push_back({c, std::move(s)});
      }
      const size_t threshold = match_limit << times_banned[r];
      if (ms.size() > threshold) {
        banned_until[r] = it + (ban_length << times_banned[r]);
        ++times_banned[r];
        continue;
      }
      found.push_back({r, std::move(ms)});
    }
    bool changed = false;
    for (auto& [r, ms] : found) {
      for (auto& [c, s] : ms) {
        const uint32_t target = eg.find(c);
        const Info want = eg.cls[target].data;
        const Info got = rhs_info(eg, rules[r].rhs, s);
        if (!got.valid || got.shape != want.shape || got.dtype != want.dtype) continue;
        uint32_t id = instantiate(eg, rules[r].rhs, s);
        changed = eg.merge(target, id) || changed;
        if (eg.n_nodes > node_limit) break;
      }
      if (eg.n_nodes > node_limit) break;
    }
    eg.rebuild();
    if (eg.n_nodes > node_limit) {
      ++it;
      break;
    }
    bool any_banned = false;
    for (size_t r = 0; r < rules.size(); ++r) any_banned = any_banned || banned_until[r] > it + 1;
    if (!changed && !any_banned) {
      ++it;
      break;
    }
  }
  st->iterations = it;
  st->egraph_nodes = eg.n_nodes;

  // Tree-cost extraction: each class's cheapest node, children counted per use.
  const double INF = std::numeric_limits<double>::infinity();
  std::vector<double> best(eg.cls.size(), INF);
  std::vector<int> choice(eg.cls.size(), -1);
  auto node_cost = [&](const ENode& n, const Info& data) -> double {
    if (n.sym == Sym::Leaf) return 0.0;
    std::vector<const Info*> kids;
    bool all_const = !n.kids.empty();
    for (auto k : n.kids) {
      const Info& ki = eg.cls[eg.find(k)].data;
      if (!ki.valid) return INF;
      kids.push_back(&ki);
      all_const = all_const && ki.splat.has_value();
    }
    double own = 0.0;
    if (!all_const) {
      std::vector<const std::vector<size_t>*> args;
      for (auto* k : kids) args.push_back(&k->shape);
      const Op op = n.sym == Sym::Opaque ? opaque_ops[n.key] : op_of_sym(n.sym);
      own = model.node(op, data.shape, args);
    }
    for (auto k : n.kids) own += best[eg.find(k)];
    return own;
  };
  for (bool progress = true; progress;) {
    progress = false;
    for (uint32_t c = 0; c < eg.cls.size(); ++c) {
      if (eg.find(c) != c || !eg.cls[c].data.valid) continue;
      for (size_t q = 0; q < eg.cls[c].nodes.size(); ++q) {
        double v = node_cost(eg.cls[c].nodes[q], eg.cls[c].data);
        if (v < best[c]) {
          best[c] = v;
          choice[c] = (int)q;
          progress = true;
        }
      }
    }
  }

  // Rebuild a graph from the choices: inputs first so their numbering survives; sources and
  // backward marks follow the class (a class computed in the forward pass stays there).
  std::map<uint32_t, std::pair<std::shared_ptr<const std::string>, bool>> role;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!keep[i] && g.nodes[i].op.kind != OpKind::Input) continue;
    uint32_t c = eg.find(cls_of[i]);
    auto ins = role.emplace(c, std::make_pair(g.nodes[i].source, g.nodes[i].origin.has_value()));
    if (!ins.second) ins.first->second.second = ins.first->second.second && g.nodes[i].origin.has_value();
  }
  Graph h;
  std::map<uint32_t, uint32_t> built;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (g.nodes[i].op.kind != OpKind::Input) continue;
    h.cur_source = g.nodes[i].source;
    uint32_t id = h.input(g.nodes[i].shape, g.nodes[i].dtype);
    h.nodes[id].op = g.nodes[i].op;
    built[eg.find(cls_of[i])] = id;
  }
  std::vector<uint32_t> roots(outputs.begin(), outputs.end());
  std::map<uint32_t, bool> on_path;
  for (uint32_t root : roots) {
    std::vector<uint32_t> stack = {eg.find(cls_of[root])};
    while (!stack.empty()) {
      uint32_t c = stack.back();
      if (built.count(c)) {
        stack.pop_back();
        on_path.erase(c);
        continue;
      }
      if (choice[c] < 0) return std::nullopt;
      const ENode& n = eg.cls[c].nodes[(size_t)choice[c]];
      std::vector<uint32_t> missing;
      for (auto k : n.kids)
        if (!built.count(eg.find(k))) missing.push_back(eg.find(k));
      if (!missing.empty()) {
        if (on_path[c]) return std::nullopt;  // the choice has a cycle
        on_path[c] = true;
        for (auto m : missing)
          if (on_path.count(m) && on_path[m]) return std::nullopt;
        stack.insert(stack.end(), missing.begin(), missing.end());
        continue;
      }
      std::shared_ptr<const std::string> source;
      bool backward = false;
      auto r = role.find(c);
      if (r != role.end()) {
        source = r->second.first;
        backward = r->second.second;
      } else {
        // A form absent from the source inherits from its operands.
        for (auto k : n.kids) {
          auto rk = role.find(eg.find(k));
          if (rk != role.end()) {
            backward = backward || rk->second.second;
            if (!source) source = rk->second.first;
          }
        }
      }
      h.cur_source = source;
      uint32_t id;
      if (n.sym == Sym::Leaf) {
        const Node& src = g.nodes[leaf_node[n.key]];
        id = h.constant(src.op.value);
      } else {
        std::vector<uint32_t> ins;
        for (auto k : n.kids) ins.push_back(built[eg.find(k)]);
        const Op op = n.sym == Sym::Opaque ? opaque_ops[n.key] : op_of_sym(n.sym);
        try {
          id = h.add(op, ins);
        } catch (...) {
          return std::nullopt;
        }
      }
      if (backward) h.nodes[id].origin = 0;
      built[c] = id;
      on_path.erase(c);
      stack.pop_back();
    }
  }
  std::vector<uint32_t> out;
  for (auto o : outputs) out.push_back(built[eg.find(cls_of[o])]);
  return std::make_pair(std::move(h), std::move(out));
}

}  // namespace rg
