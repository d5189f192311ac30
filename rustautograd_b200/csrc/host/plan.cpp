// Plan construction: scheduling, fusion and slot allocation. Restates src/plan.rs:184-655; the
// allocation order (free-list choice, in-place release before allocation) is kept exactly so
// that the same graph yields the same slot layout as rg's planner.
#include "plan.h"

#include <algorithm>
#include <set>
#include <stdexcept>
#include <unordered_set>

namespace rg {

namespace {

// plan.rs:170-238
struct Allocator {
  std::vector<std::pair<DType, size_t>> slots;
  std::vector<bool> pinned;
  std::vector<uint32_t> refs;
  std::vector<size_t> free;
  bool reuse = true;
  std::vector<size_t> held;
  size_t live = 0, peak = 0;

  size_t new_slot(DType d, size_t n, bool pin) {
    slots.emplace_back(d, n);
    pinned.push_back(pin);
    refs.push_back(1);
    held.push_back(0);
    return slots.size() - 1;
  }
  size_t alloc(DType d, size_t n) {
    size_t s = pick(d, n);
    held[s] = n * dtype_size(d);
    live += held[s];
    peak = std::max(peak, live);
    return s;
  }
  size_t pick(DType d, size_t n) {
    // First free slot of the smallest fitting capacity; a small value may not pin a buffer more
    // than 4x its size (plan.rs:209-214).
    size_t best = SIZE_MAX, best_cap = 0;
    for (size_t k = 0; k < free.size(); ++k) {
      size_t s = free[k];
      if (slots[s].first == d && slots[s].second >= n && slots[s].second <= std::max<size_t>(n, 1) * 4) {
        if (best == SIZE_MAX || slots[s].second < best_cap) {
          best = k;
          best_cap = slots[s].second;
        }
      }
    }
    if (best != SIZE_MAX) {
      size_t s = free[best];
      free[best] = free.back();  // Vec::swap_remove
      free.pop_back();
      refs[s] = 1;
      return s;
    }
    return new_slot(d, n, false);
  }
  void release(size_t s) {
    refs[s] -= 1;
    if (refs[s] == 0 && !pinned[s]) {
      live -= held[s];
      if (reuse) free.push_back(s);
    }
  }
};

constexpr size_t LEVEL_ORDER_MAX_PEAK = size_t(2) << 30;

bool arg_kind(const std::vector<size_t>& s, const std::vector<size_t>& shape, ArgKind* k, size_t* row) {
  size_t n = product(s);
  if (s == shape) {
    *k = ArgKind::Full;
  } else if (n == 1) {
    *k = ArgKind::Splat;
  } else if (!s.empty() && !shape.empty() && s.back() == shape.back() && n == s.back()) {
    *k = ArgKind::Row;
    *row = n;
  } else {
    return false;
  }
  return true;
}

double op_cost_ns(const Op& op) {
  switch (op.kind) {
    case OpKind::Exp: case OpKind::Log: case OpKind::Sin: case OpKind::Cos: case OpKind::Tanh: return 0.6;
    case OpKind::Pow: return 10.0;
    case OpKind::Div: case OpKind::Sqrt: return 0.2;
    default: return 0.06;
  }
}

bool fusable(const Graph& g, size_t id, bool gpu) {
  const Node& n = g.nodes[id];
  bool elementwise = n.op.is_unary_elementwise() || n.op.is_binary_elementwise() || n.op.kind == OpKind::Where;
  if (!elementwise || n.dtype == DType::I32) return false;
  if (gpu) return true;
  for (auto x : n.inputs) {
    ArgKind k;
    size_t r;
    if (!arg_kind(g.shape(x), n.shape, &k, &r)) return false;
  }
  return true;
}

// plan.rs:285-295
bool metal_on_cpu(const Op& op, DType dtype, size_t n, const std::vector<DType>& args) {
  bool wide = dtype == DType::F64 || std::find(args.begin(), args.end(), DType::F64) != args.end();
  bool small_int = dtype == DType::I32 && n <= 64 && std::all_of(args.begin(), args.end(), [](DType d) { return d == DType::I32; });
  return wide || small_int || op.kind == OpKind::RandNormal || op.kind == OpKind::KeySplit;
}

bool is_leaf(const Node& n) { return n.op.kind == OpKind::Input || n.op.kind == OpKind::Const; }

std::vector<bool> hoisted(const Graph& g, const std::vector<bool>& keep) {
  std::vector<bool> up(g.nodes.size(), false);
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    if (!keep[i] || is_leaf(n)) continue;
    bool ready = true;
    for (auto x : n.inputs) ready = ready && (up[x] || is_leaf(g.nodes[x]));
    std::vector<DType> dts;
    for (auto x : n.inputs) dts.push_back(g.dtype(x));
    bool all_up = true;
    for (auto x : n.inputs) all_up = all_up && up[x];
    up[i] = ready && (metal_on_cpu(n.op, n.dtype, n.n(), dts) || (is_alias(g, i) && all_up));
  }
  return up;
}

struct Item {
  bool group = false;
  size_t node = 0;
  std::vector<size_t> members;
};

bool contains(const std::vector<size_t>& v, size_t x) { return std::find(v.begin(), v.end(), x) != v.end(); }

size_t external_inputs(const Graph& g, const std::vector<size_t>& members, const Node& extra) {
  std::unordered_set<uint32_t> s;
  for (size_t m : members)
    for (auto x : g.nodes[m].inputs)
      if (!contains(members, x)) s.insert(x);
  for (auto x : extra.inputs)
    if (!contains(members, x)) s.insert(x);
  return s.size();
}

std::vector<Item> schedule_levels(const Graph& g, const std::vector<bool>& keep, const Fuse& cfg);

// Fuse::hoist_small: tiny elementwise, cast and key-split nodes whose inputs are leaves or
// themselves hoisted.
std::vector<bool> hoisted_small(const Graph& g, const std::vector<bool>& keep) {
  std::vector<bool> up(g.nodes.size(), false);
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    if (!keep[i] || is_leaf(n) || n.n() > 64) continue;
    const OpKind k = n.op.kind;
    bool kind_ok = n.op.is_unary_elementwise() || n.op.is_binary_elementwise() || k == OpKind::Where || k == OpKind::Cast || k == OpKind::KeySplit;
    if (!kind_ok) continue;
    bool ready = true;
    for (auto x : n.inputs) ready = ready && (up[x] || is_leaf(g.nodes[x]));
    up[i] = ready;
  }
  return up;
}

std::vector<bool> hoisted_for(const Graph& g, const std::vector<bool>& keep, const Fuse& cfg) {
  if (cfg.gpu && cfg.hoist) return hoisted(g, keep);
  if (cfg.hoist_small) return hoisted_small(g, keep);
  return std::vector<bool>(g.nodes.size(), false);
}

// Emits the hoisted nodes first, in graph order. Under hoist_small, consecutive fusable nodes of
// one shape and dtype become one group (a scalar chain runs as a single kernel).
void emit_hoisted(const Graph& g, const std::vector<bool>& up, const Fuse& cfg, std::vector<Item>& items) {
  std::vector<size_t> open;
  auto close = [&]() {
    if (open.size() >= 2) {
      Item it;
      it.group = true;
      it.members = open;
      items.push_back(std::move(it));
    } else {
      for (size_t m : open) items.push_back(Item{false, m, {}});
    }
    open.clear();
  };
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!up[i]) continue;
    const Node& n = g.nodes[i];
    if (cfg.hoist_small && fusable(g, i, true)) {
      bool same = open.empty() || (g.nodes[open[0]].shape == n.shape && g.nodes[open[0]].dtype == n.dtype);
      if (!same || external_inputs(g, open, n) + open.size() + 1 > cfg.max_bindings) close();
      open.push_back(i);
    } else {
      bool reads_open = false;
      for (auto x : n.inputs) reads_open = reads_open || contains(open, x);
      if (reads_open) close();
      items.push_back(Item{false, i, {}});
    }
  }
  close();
}

// Device plans with data parallelism (no counterpart in rg): the all-reduces and every node that
// depends on one (the optimizer update, the reported loss) come after all other nodes, so the
// all-reduces are consecutive plan steps that run as one NCCL group after the backward pass,
// instead of one group per gradient between pieces of it (each group a synchronisation point).
std::vector<bool> after_collectives(const Graph& g, const std::vector<bool>& keep, const Fuse& cfg) {
  std::vector<bool> late(g.nodes.size(), false);
  if (!cfg.gpu) return late;
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!keep[i]) continue;
    const Node& n = g.nodes[i];
    bool dep = n.op.kind == OpKind::AllReduce;
    for (auto x : n.inputs) dep = dep || late[x];
    late[i] = dep;
  }
  return late;
}

// plan.rs:297-350
std::vector<Item> schedule(const Graph& g, const std::vector<bool>& keep, const Fuse& cfg) {
  if (cfg.gpu && cfg.levels) return schedule_levels(g, keep, cfg);
  std::vector<Item> items;
  std::vector<size_t> open;
  auto close = [&]() {
    double cost = 0;
    for (size_t m : open) cost += op_cost_ns(g.nodes[m].op) * (double)g.nodes[m].n();
    if (open.size() >= (cfg.gpu ? 2u : 1u) && cost >= cfg.parallel_ns) {
      Item it;
      it.group = true;
      it.members = std::move(open);
      items.push_back(std::move(it));
    } else {
      for (size_t m : open) items.push_back(Item{false, m, {}});
    }
    open.clear();
  };
  std::vector<bool> up = hoisted_for(g, keep, cfg);
  emit_hoisted(g, up, cfg, items);
  const std::vector<bool> late = after_collectives(g, keep, cfg);
  // Passes: the nodes before any all-reduce, the all-reduces, what depends on them.
  for (int pass = 0; pass < 3; ++pass) {
    for (size_t i = 0; i < g.nodes.size(); ++i) {
      const Node& n = g.nodes[i];
      if (!keep[i] || up[i] || is_leaf(n)) continue;
      const int want = !late[i] ? 0 : n.op.kind == OpKind::AllReduce ? 1 : 2;
      if (want != pass) continue;
      if (fusable(g, i, cfg.gpu) && !(cfg.hoist && n.dtype == DType::F64)) {
        bool same = open.empty() || (g.nodes[open[0]].shape == n.shape && g.nodes[open[0]].dtype == n.dtype);
        size_t inputs = external_inputs(g, open, n);
        if (!same || (cfg.gpu && inputs + open.size() + 1 > cfg.max_bindings)) close();
        open.push_back(i);
      } else {
        bool reads_open = false;
        for (auto x : n.inputs) reads_open = reads_open || contains(open, x);
        if (reads_open) close();
        items.push_back(Item{false, i, {}});
      }
    }
    close();
  }
  return items;
}

// plan.rs:352-414: every node gets a dependency level; a level holds one group per shape.
std::vector<Item> schedule_levels(const Graph& g, const std::vector<bool>& keep, const Fuse& cfg) {
  std::vector<bool> up = hoisted_for(g, keep, cfg);
  std::vector<Item> items;
  emit_hoisted(g, up, cfg, items);
  auto gpu_fusable = [&](size_t i) { return fusable(g, i, true) && !(cfg.hoist && g.nodes[i].dtype == DType::F64); };
  std::vector<size_t> level(g.nodes.size(), 0);
  std::vector<std::vector<size_t>> by_level;
  // The all-reduces and what depends on them go above every other node, the all-reduces on one
  // level (after_collectives).
  const std::vector<bool> late = after_collectives(g, keep, cfg);
  size_t top = 0;
  for (int pass = 0; pass < 2; ++pass)
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    const Node& n = g.nodes[i];
    if (!keep[i] || up[i] || is_leaf(n) || late[i] != (pass == 1)) continue;
    if (n.op.kind == OpKind::AllReduce) {
      level[i] = top + 1;
      continue;
    }
    size_t deepest = 0;
    for (auto x : n.inputs) deepest = std::max(deepest, level[x]);
    bool joins = gpu_fusable(i) && deepest > 0;
    if (joins) {
      for (auto x : n.inputs) {
        if (!(level[x] < deepest || (gpu_fusable(x) && g.nodes[x].shape == n.shape && g.nodes[x].dtype == n.dtype))) {
          joins = false;
          break;
        }
      }
    }
    level[i] = (is_alias(g, i) || joins) ? deepest : deepest + 1;
    if (pass == 0) top = std::max(top, level[i]);
  }
  if (cfg.sink) {
    // Consumers first (reverse graph order), so that a chain of such nodes follows its last link.
    // The new level is above every input's, so the node's inputs are still computed before it.
    std::vector<std::vector<size_t>> users(g.nodes.size());
    for (size_t i = 0; i < g.nodes.size(); ++i)
      if (keep[i] && !up[i] && !is_leaf(g.nodes[i]))
        for (auto x : g.nodes[i].inputs) users[x].push_back(i);
    for (size_t i = g.nodes.size(); i-- > 0;) {
      const Node& n = g.nodes[i];
      if (!keep[i] || up[i] || is_leaf(n) || is_alias(g, i) || !gpu_fusable(i) || users[i].empty()) continue;
      size_t first = SIZE_MAX;
      bool all = true;
      for (size_t u : users[i]) {
        const Node& c = g.nodes[u];
        all = all && !is_alias(g, u) && gpu_fusable(u) && c.shape == n.shape && c.dtype == n.dtype;
        first = std::min(first, level[u]);
      }
      if (all && first > level[i]) level[i] = first;
    }
  }
  for (size_t i = 0; i < g.nodes.size(); ++i) {
    if (!keep[i] || up[i] || is_leaf(g.nodes[i])) continue;
    if (by_level.size() <= level[i]) by_level.resize(level[i] + 1);
    by_level[level[i]].push_back(i);
  }
  for (auto& nodes : by_level) {
    std::vector<std::vector<size_t>> groups;
    std::vector<size_t> aliases;
    for (size_t i : nodes) {
      const Node& n = g.nodes[i];
      if (is_alias(g, i)) {
        aliases.push_back(i);
      } else if (gpu_fusable(i)) {
        ptrdiff_t found = -1;
        for (size_t k = groups.size(); k-- > 0;) {
          const Node& f = g.nodes[groups[k][0]];
          if (f.shape == n.shape && f.dtype == n.dtype) {
            found = (ptrdiff_t)k;
            break;
          }
        }
        bool fits = found >= 0 && external_inputs(g, groups[found], n) + groups[found].size() + 1 <= cfg.max_bindings;
        if (found >= 0 && fits) groups[found].push_back(i);
        else groups.push_back({i});
      } else {
        items.push_back(Item{false, i, {}});
      }
    }
    for (auto& m : groups) {
      if (m.size() >= 2) {
        Item it;
        it.group = true;
        it.members = m;
        items.push_back(std::move(it));
      } else {
        for (size_t x : m) items.push_back(Item{false, x, {}});
      }
    }
    for (size_t a : aliases) items.push_back(Item{false, a, {}});
  }
  return items;
}

// plan.rs:416-457
Fused compile_group(const Graph& g, const std::vector<size_t>& members, const std::vector<size_t>& slot_of,
                    const std::vector<std::pair<size_t, size_t>>& out_slots) {
  const Node& first = g.nodes[members[0]];
  Fused f;
  std::vector<std::pair<uint32_t, Operand>> ext;
  size_t regs = 0;
  for (size_t m : members) {
    for (auto x : g.nodes[m].inputs) {
      if (contains(members, x)) continue;
      bool seen = false;
      for (auto& e : ext) seen = seen || e.first == x;
      if (seen) continue;
      ArgKind kind = ArgKind::Broadcast;
      size_t row = 0;
      if (!arg_kind(g.shape(x), first.shape, &kind, &row)) kind = ArgKind::Broadcast;
      f.input_shapes.push_back(g.shape(x));
      Operand operand;
      if (kind == ArgKind::Full) {
        operand = Operand{false, f.inputs.size()};
      } else {
        regs += 1;
        operand = Operand{true, regs - 1};
      }
      FusedInput in;
      in.slot = slot_of[x];
      in.kind = kind;
      in.row = row;
      in.reg = operand.reg ? operand.idx : SIZE_MAX;
      f.inputs.push_back(in);
      ext.emplace_back(x, operand);
    }
  }
  std::vector<size_t> reg_of(g.nodes.size(), SIZE_MAX);
  for (size_t m : members) {
    MicroOp mo;
    mo.op = g.nodes[m].op;
    for (auto x : g.nodes[m].inputs) {
      bool found = false;
      for (auto& e : ext) {
        if (e.first == x) {
          mo.args.push_back(e.second);
          found = true;
          break;
        }
      }
      if (!found) mo.args.push_back(Operand{true, reg_of[x]});
    }
    reg_of[m] = regs;
    mo.reg = regs;
    f.ops.push_back(std::move(mo));
    regs += 1;
  }
  for (auto& os : out_slots) f.outputs.emplace_back(reg_of[os.first], os.second);
  f.dtype = first.dtype;
  f.n = first.n();
  f.regs = regs;
  f.shape = first.shape;
  return f;
}

}  // namespace

bool is_alias(const Graph& g, size_t id) {
  const Node& n = g.nodes[id];
  switch (n.op.kind) {
    case OpKind::Reshape: case OpKind::StopGradient: case OpKind::Custom: return true;
    case OpKind::Cast: return n.op.dtype == g.nodes[n.inputs[0]].dtype;
    default: return false;
  }
}

std::vector<size_t> strides(const std::vector<size_t>& shape) {
  std::vector<size_t> out(shape.size(), 1);
  for (size_t i = shape.size() > 0 ? shape.size() - 1 : 0; i-- > 0;) out[i] = out[i + 1] * shape[i + 1];
  return out;
}

std::vector<size_t> bstrides(const std::vector<size_t>& shape, size_t rank) {
  auto st = strides(shape);
  size_t lead = rank - shape.size();
  std::vector<size_t> out(rank, 0);
  for (size_t i = 0; i < rank; ++i) out[i] = (i < lead || shape[i - lead] == 1) ? 0 : st[i - lead];
  return out;
}

// plan.rs:1034-1050
Mode binary_mode(const Op& op, const std::vector<size_t>& shape, const std::vector<std::vector<size_t>>& args) {
  if (!op.is_binary_elementwise()) return Mode::Same;
  const auto &a = args[0], &b = args[1];
  if (a == shape && b == shape) return Mode::Same;
  if (product(a) == 1 && b == shape) return Mode::AScalar;
  if (a == shape && product(b) == 1) return Mode::BScalar;
  return Mode::General;
}

Plan Plan::build(const Graph& g, const std::vector<uint32_t>& outputs, bool reuse) {
  return build_with(g, outputs, reuse, nullptr);
}

Plan Plan::build_fused(const Graph& g, const std::vector<uint32_t>& outputs, const Fuse& cfg) {
  Plan plan = build_with(g, outputs, true, &cfg);
  if (!(cfg.gpu && cfg.levels)) return plan;
  // Level order cuts launches but keeps values alive longer (plan.rs:470-478).
  Fuse greedy_cfg = cfg;
  greedy_cfg.levels = false;
  Plan greedy = build_with(g, outputs, true, &greedy_cfg);
  if (plan.peak_live_bytes > LEVEL_ORDER_MAX_PEAK || greedy.gpu_cost_estimate() < plan.gpu_cost_estimate()) {
    greedy.fuse = cfg;
    return greedy;
  }
  return plan;
}

double Plan::gpu_cost_estimate() const {
  const double PER_DISPATCH_NS = 30000.0, PER_ELEMENT_NS = 0.1;
  double c = 0;
  for (auto& s : steps) {
    if (s.fused) c += PER_DISPATCH_NS + PER_ELEMENT_NS * (double)(s.group.n * s.group.outputs.size());
    else c += PER_DISPATCH_NS + PER_ELEMENT_NS * (double)s.instr.n;
  }
  return c;
}

size_t Plan::planned_bytes() const {
  size_t b = 0;
  for (size_t i = 0; i < slots.size(); ++i)
    if (!pinned[i]) b += dtype_size(slots[i].first) * slots[i].second;
  return b;
}

size_t Plan::n_fused() const {
  size_t k = 0;
  for (auto& s : steps) k += s.fused;
  return k;
}

size_t Plan::n_fused_ops() const {
  size_t k = 0;
  for (auto& s : steps)
    if (s.fused) k += s.group.ops.size();
  return k;
}

// plan.rs:502-634
Plan Plan::build_with(const Graph& g, const std::vector<uint32_t>& outputs, bool reuse, const Fuse* fuse) {
  auto keep = g.reachable(outputs);
  size_t total = g.nodes.size();
  std::vector<uint32_t> uses(total, 0);
  for (size_t i = 0; i < total; ++i)
    if (keep[i])
      for (auto x : g.nodes[i].inputs) uses[x] += 1;
  for (auto o : outputs) uses[o] += 1;

  Allocator a;
  a.reuse = reuse;
  std::vector<size_t> value_slot(total, SIZE_MAX);
  Plan p;
  p.input_slots.assign(g.n_inputs, 0);
  p.input_ns.assign(g.n_inputs, 0);

  for (size_t i = 0; i < total; ++i) {
    const Node& node = g.nodes[i];
    if (node.op.kind == OpKind::Input) {
      size_t s = a.new_slot(node.dtype, node.n(), true);
      p.input_slots[node.op.index] = s;
      p.input_ns[node.op.index] = node.n();
      value_slot[i] = s;
    } else if (node.op.kind == OpKind::Const && keep[i]) {
      size_t s = a.new_slot(node.dtype, node.n(), true);
      p.consts.emplace_back(s, node.op.value);
      value_slot[i] = s;
    }
  }

  std::vector<Item> items;
  if (fuse) {
    items = schedule(g, keep, *fuse);
  } else {
    for (size_t i = 0; i < total; ++i)
      if (keep[i] && !is_leaf(g.nodes[i])) items.push_back(Item{false, i, {}});
  }

  for (auto& item : items) {
    if (item.group) {
      const auto& members = item.members;
      std::vector<uint32_t> external;
      for (size_t m : members) {
        p.naive_bytes += g.nodes[m].n() * dtype_size(g.nodes[m].dtype);
        for (auto x : g.nodes[m].inputs) {
          uses[x] -= 1;
          if (!contains(members, x) && std::find(external.begin(), external.end(), x) == external.end()) external.push_back(x);
        }
      }
      // Destinations first, so they never share a buffer with an input.
      std::vector<std::pair<size_t, size_t>> out_slots;
      for (size_t m : members) {
        if (uses[m] > 0) {
          size_t s = a.alloc(g.nodes[m].dtype, g.nodes[m].n());
          value_slot[m] = s;
          out_slots.emplace_back(m, s);
        }
      }
      Step st;
      st.fused = true;
      st.group = compile_group(g, members, value_slot, out_slots);
      p.steps.push_back(std::move(st));
      for (auto x : external)
        if (uses[x] == 0) a.release(value_slot[x]);
      continue;
    }
    size_t i = item.node;
    const Node& node = g.nodes[i];
    if (node.op.kind == OpKind::Output) continue;  // allocated with its control-flow step
    if (is_alias(g, i)) {
      size_t x = node.inputs[0];
      size_t s = value_slot[x];
      a.refs[s] += 1;
      value_slot[i] = s;
      uses[x] -= 1;
      if (uses[x] == 0) a.release(s);
      continue;
    }
    Instr ins;
    for (auto x : node.inputs) {
      ins.arg_shapes.push_back(g.shape(x));
      ins.args.push_back(value_slot[x]);
    }
    ins.mode = binary_mode(node.op, node.shape, ins.arg_shapes);
    for (auto x : node.inputs) uses[x] -= 1;
    std::vector<uint32_t> dying;
    for (auto x : node.inputs)
      if (uses[x] == 0) dying.push_back(x);
    std::sort(dying.begin(), dying.end());
    dying.erase(std::unique(dying.begin(), dying.end()), dying.end());
    bool elementwise = node.op.is_unary_elementwise() || node.op.is_binary_elementwise();
    auto inplace = [&](uint32_t x) {
      return elementwise && ins.mode != Mode::General && g.shape(x) == node.shape && g.dtype(x) == node.dtype;
    };
    for (auto x : dying)
      if (inplace(x)) a.release(value_slot[x]);
    size_t dst;
    if (node.op.is_control_flow()) {
      for (size_t o = 0; o < total; ++o) {
        const Node& out = g.nodes[o];
        if (keep[o] && out.op.kind == OpKind::Output && !out.inputs.empty() && out.inputs[0] == i) {
          size_t slot = a.alloc(out.dtype, out.n());
          value_slot[o] = slot;
          ins.outs.emplace_back(out.op.index, slot);
        }
      }
      dst = SIZE_MAX;
    } else {
      dst = a.alloc(node.dtype, node.n());
    }
    for (auto x : dying)
      if (!inplace(x)) a.release(value_slot[x]);
    value_slot[i] = dst;
    p.naive_bytes += node.n() * dtype_size(node.dtype);
    if (node.op.is_control_flow()) {
      // plan.rs:714-719: reference plans run reference bodies, everything else the fast ones.
      Fuse body_cfg = fuse ? *fuse : Fuse::DEFAULT();
      ins.body_plan = reuse ? node.op.body->plan_for(body_cfg) : node.op.body->reference;
      if (node.op.body2) ins.body2_plan = reuse ? node.op.body2->plan_for(body_cfg) : node.op.body2->reference;
    }
    ins.op = node.op;
    ins.node = (uint32_t)i;
    ins.dtype = node.dtype;
    ins.dst = dst;
    ins.shape = node.shape;
    ins.n = node.n();
    Step st;
    st.fused = false;
    st.instr = std::move(ins);
    p.steps.push_back(std::move(st));
  }

  for (auto o : outputs) p.outputs.push_back(PlanOutput{value_slot[o], g.shape(o), g.nodes[o].n()});
  p.reference = !reuse;
  p.slots = std::move(a.slots);
  p.pinned = std::move(a.pinned);
  p.peak_live_bytes = a.peak;
  p.fuse = fuse ? *fuse : Fuse::DEFAULT();
  return p;
}

static EvalFn g_eval;

void set_evaluator(EvalFn f) { g_eval = std::move(f); }
bool has_evaluator() { return (bool)g_eval; }

std::vector<Tensor> eval(const Graph& g, const std::vector<uint32_t>& outputs, const std::vector<const Tensor*>& inputs) {
  if (!g_eval) throw std::runtime_error("no device is installed to evaluate graphs in this process");
  Plan plan = Plan::build(g, outputs, true);
  return g_eval(plan, inputs);
}

}  // namespace rg
