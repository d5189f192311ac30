// Row chains (rowchain.h): which plan steps one row kernel computes, what it writes, and which
// other steps of the range move before or after it.
#include "rowchain.h"

#include <algorithm>
#include <cstdlib>
#include <map>
#include <string>

namespace rg {

// On by default; RGC_ROW_CHAINS=0 runs every step of a chain as its own kernel (the results are
// the same bits either way).
bool row_chains_enabled() {
  const char* e = getenv("RGC_ROW_CHAINS");
  return !(e && std::string(e) == "0");
}

std::vector<size_t> step_reads(const Step& s) {
  std::vector<size_t> r;
  if (s.fused) {
    for (auto& in : s.group.inputs) r.push_back(in.slot);
  } else {
    r = s.instr.args;
  }
  return r;
}

std::vector<size_t> step_writes(const Step& s) {
  std::vector<size_t> w;
  if (s.fused) {
    for (auto& o : s.group.outputs) w.push_back(o.second);
  } else {
    if (s.instr.dst != SIZE_MAX) w.push_back(s.instr.dst);
    for (auto& o : s.instr.outs) w.push_back(o.second);
  }
  return w;
}

namespace {

enum class Role { None, Full, Col, Reduce };

// Rows up to this length fit a block of rows in shared memory.
constexpr size_t MAX_COLS_F32 = 1024, MAX_COLS_F64 = 512;
// Full-size values a chain keeps in shared memory between its stages, and per-row values.
constexpr size_t MAX_BUFFERS = 4, MAX_COLUMNS = 32;
// Kernel parameters: slots read and slots written.
constexpr size_t MAX_BINDINGS = 64;
// Non-member steps scanned past the last member before the chain is closed.
constexpr size_t LOOKAHEAD = 6;

bool elementwise(const Instr& i) { return i.op.is_unary_elementwise() || i.op.is_binary_elementwise() || i.op.kind == OpKind::Where; }

std::vector<size_t> per_row(std::vector<size_t> s) {
  s.back() = 1;
  return s;
}

std::vector<size_t> strip_ones(const std::vector<size_t>& s) {
  size_t k = 0;
  while (k + 1 < s.size() && s[k] == 1) ++k;
  return std::vector<size_t>(s.begin() + (long)k, s.end());
}

// `as` (leading ones aside) is a trailing part of `shape`: element e reads e mod product(as).
bool is_suffix(const std::vector<size_t>& as, const std::vector<size_t>& shape) {
  auto a = strip_ones(as);
  if (a.size() > shape.size()) return false;
  return std::equal(a.begin(), a.end(), shape.end() - (long)a.size());
}

Role role_of(const Step& st, const std::vector<size_t>& S, DType dt) {
  const auto Sc = per_row(S);
  if (st.fused) {
    const Fused& g = st.group;
    if (g.dtype != dt) return Role::None;
    if (g.shape == S) return Role::Full;
    if (g.shape == Sc) return Role::Col;
    return Role::None;
  }
  const Instr& i = st.instr;
  if (i.dtype != dt) return Role::None;
  if (elementwise(i)) {
    if (i.shape == S) return Role::Full;
    if (i.shape == Sc) return Role::Col;
    return Role::None;
  }
  if (i.op.kind == OpKind::Reduce && i.args.size() == 1 && i.arg_shapes[0] == S && i.shape == Sc && i.op.shape.size() == 1 &&
      i.op.shape[0] == S.size() - 1)
    return Role::Reduce;
  return Role::None;
}

// Input slots and their shapes, in input order.
std::vector<std::pair<size_t, std::vector<size_t>>> inputs_of(const Step& st) {
  std::vector<std::pair<size_t, std::vector<size_t>>> r;
  if (st.fused) {
    for (size_t k = 0; k < st.group.inputs.size(); ++k) r.push_back({st.group.inputs[k].slot, st.group.input_shapes[k]});
  } else {
    for (size_t k = 0; k < st.instr.args.size(); ++k) r.push_back({st.instr.args[k], st.instr.arg_shapes[k]});
  }
  return r;
}

const std::vector<size_t>& shape_of(const Step& st) { return st.fused ? st.group.shape : st.instr.shape; }

bool contains(const std::vector<size_t>& v, size_t x) { return std::find(v.begin(), v.end(), x) != v.end(); }

struct Builder {
  Builder(const Plan& p, std::vector<size_t> shape, DType d) : plan(p), S(shape), Sc(shape.empty() ? shape : per_row(shape)), dt(d) {}
  const Plan& plan;
  std::vector<size_t> S, Sc;
  DType dt = DType::F32;
  RowChain c;
  std::vector<Role> roles;                                   // per member
  std::map<size_t, std::pair<size_t, size_t>> latest;        // slot -> (member, output) last written
  std::vector<size_t> member_writes, member_reads, after_writes, after_reads;
  // Slots members read in place of a broadcast of them: no later step of the chain may write them.
  std::vector<size_t> sources;
  std::map<size_t, bool> external_row_local;                 // slot read from outside: every read row-local

  // The plan step that last wrote `slot` before step `p`, or SIZE_MAX.
  size_t last_writer(size_t slot, size_t p) const {
    for (size_t q = p; q-- > 0;)
      if (contains(step_writes(plan.steps[q]), slot)) return q;
    return SIZE_MAX;
  }

  // A materialised broadcast (step `step`) of a slot of the same dtype that still holds the
  // broadcast's source when step `p` reads it: a pinned slot, or one no step in between writes.
  // Its source slot, else SIZE_MAX.
  size_t broadcast_source(size_t step, size_t p) const {
    if (step == SIZE_MAX) return SIZE_MAX;
    const Step& w = plan.steps[step];
    if (w.fused || w.instr.op.kind != OpKind::BroadcastTo || w.instr.args.size() != 1) return SIZE_MAX;
    size_t src = w.instr.args[0];
    if (src >= plan.pinned.size() || plan.slots[src].first != w.instr.dtype) return SIZE_MAX;
    if (!plan.pinned[src])
      for (size_t q = step + 1; q < p; ++q)
        if (contains(step_writes(plan.steps[q]), src)) return SIZE_MAX;
    return src;
  }

  bool classify(size_t p, Role r, std::vector<RowInput>* out) const {
    const Step& st = plan.steps[p];
    const auto& shape = shape_of(st);
    for (auto& [slot, as] : inputs_of(st)) {
      if (plan.slots[slot].first != dt) return false;
      RowInput in;
      in.slot = slot;
      auto it = latest.find(slot);
      if (it != latest.end()) {
        in.kind = RowInput::Value;
        in.producer = it->second.first;
        in.output = it->second.second;
        in.full_space = roles[in.producer] == Role::Full;
        bool ok = r == Role::Reduce ? (in.full_space && as == S)
                  : r == Role::Full ? (in.full_space ? as == S : as == Sc)
                                    : (!in.full_space && as == Sc);
        if (!ok) return false;
        out->push_back(in);
        continue;
      }
      in.shape = as;
      if (r == Role::Reduce) {
        if (as != S) return false;
        in.kind = RowInput::Full;
      } else if (as == shape) {
        in.kind = RowInput::Full;
        size_t src = broadcast_source(last_writer(slot, p), p);
        if (src != SIZE_MAX) {
          in.kind = RowInput::Source;
          in.through = slot;
          in.slot = src;
          in.shape = plan.steps[last_writer(slot, p)].instr.arg_shapes[0];
          if (is_suffix(in.shape, shape)) {
            size_t n = product(in.shape);
            in.kind = n == 1 ? RowInput::Splat : RowInput::Periodic;
            in.period = n;
          }
        }
      } else if (r == Role::Full && as == Sc) {
        in.kind = RowInput::Column;
      } else if (product(as) == 1) {
        in.kind = RowInput::Splat;
      } else if (is_suffix(as, shape)) {
        in.kind = RowInput::Periodic;
        in.period = product(as);
      } else {
        in.kind = RowInput::Broadcast;
      }
      out->push_back(in);
    }
    return true;
  }

  bool row_local(const RowInput& in) const { return in.kind == RowInput::Full || in.kind == RowInput::Column; }

  bool try_member(size_t p) {
    const Step& st = plan.steps[p];
    Role r = role_of(st, S, dt);
    if (r == Role::None) return false;
    std::vector<RowInput> ins;
    if (!classify(p, r, &ins)) return false;
    auto writes = step_writes(st);
    for (size_t x : writes) {
      if (plan.slots[x].first != dt || contains(sources, x)) return false;
      // Other row blocks may still read a slot that is read as a whole (not row by row).
      auto e = external_row_local.find(x);
      if (e != external_row_local.end() && !e->second) return false;
      if (contains(after_reads, x) || contains(after_writes, x)) return false;
    }
    for (auto& in : ins) {
      // A deferred broadcast has not run yet: its slot is read through its source only.
      if (in.kind != RowInput::Value && in.through == SIZE_MAX && contains(after_writes, in.slot)) return false;
    }
    size_t m = c.members.size();
    c.members.push_back(p);
    roles.push_back(r);
    for (auto& in : ins) {
      if (in.kind == RowInput::Value) continue;
      bool local = row_local(in);
      auto e = external_row_local.find(in.slot);
      if (e == external_row_local.end()) external_row_local[in.slot] = local;
      else e->second = e->second && local;
    }
    // Every slot the step names, including broadcasts read through their source: the CPU
    // interpreter that checks chain plans reads them in plan order.
    for (size_t x : step_reads(st)) member_reads.push_back(x);
    for (auto& in : ins)
      if (in.through != SIZE_MAX) sources.push_back(in.slot);
    for (size_t q = 0; q < writes.size(); ++q) {
      latest[writes[q]] = {m, q};
      member_writes.push_back(writes[q]);
    }
    return true;
  }

  bool control(const Step& st) const {
    return !st.fused && (st.instr.op.is_control_flow() || st.instr.op.kind == OpKind::AllReduce);
  }

  bool try_before(size_t p) {
    const Step& st = plan.steps[p];
    if (control(st)) return false;
    for (size_t x : step_reads(st))
      if (contains(member_writes, x) || contains(after_writes, x)) return false;
    for (size_t x : step_writes(st))
      if (contains(member_writes, x) || contains(member_reads, x) || contains(after_writes, x) || contains(after_reads, x) || contains(sources, x))
        return false;
    c.before.push_back(p);
    return true;
  }

  bool try_after(size_t p) {
    const Step& st = plan.steps[p];
    if (broadcast_source(p, p) == SIZE_MAX) return false;
    for (size_t x : step_reads(st))
      if (contains(member_writes, x)) return false;
    for (size_t x : step_writes(st)) {
      after_writes.push_back(x);
    }
    for (size_t x : step_reads(st)) after_reads.push_back(x);
    c.after.push_back(p);
    return true;
  }
};

// Members' stages: a run of full elementwise members, a run of per-row ones, or one reduction.
std::vector<int> stages(const std::vector<Role>& roles) {
  std::vector<int> s;
  int cur = -1;
  Role prev = Role::None;
  for (Role r : roles) {
    if (r != prev || r == Role::Reduce) ++cur;
    s.push_back(cur);
    prev = r;
  }
  return s;
}

std::vector<Role> roles_of(const Plan& plan, const RowChain& c) {
  std::vector<Role> r;
  for (size_t p : c.members) r.push_back(role_of(plan.steps[p], c.shape, c.dtype));
  return r;
}

// Full-size values kept in shared memory between stages: member outputs read in a later stage,
// and slots read by a reduction or in more than one stage. (The device keeps one buffer each.)
size_t buffers_needed(const Plan& plan, const RowChain& c) {
  auto roles = roles_of(plan, c);
  auto st = stages(roles);
  std::map<std::pair<size_t, size_t>, bool> values;
  std::map<size_t, std::vector<int>> slot_stages;
  std::map<size_t, bool> slot_reduced;
  for (size_t m = 0; m < c.members.size(); ++m) {
    for (auto& in : row_inputs(plan, c, m)) {
      if (in.kind == RowInput::Value && in.full_space && st[in.producer] != st[m]) values[{in.producer, in.output}] = true;
      if (in.kind == RowInput::Full && (roles[m] == Role::Full || roles[m] == Role::Reduce)) {
        slot_stages[in.slot].push_back(st[m]);
        if (roles[m] == Role::Reduce) slot_reduced[in.slot] = true;
      }
    }
  }
  size_t n = values.size();
  for (auto& [slot, ss] : slot_stages) {
    bool several = std::any_of(ss.begin(), ss.end(), [&](int s) { return s != ss[0]; });
    if (several || slot_reduced.count(slot)) ++n;
  }
  return n;
}

// Store flags and the budget check for the chain made of `c.members` (range trimmed to them).
bool finish(const Plan& plan, RowChain& c) {
  if (c.members.empty()) return false;
  c.first = c.members.front();
  c.last = c.members.back();
  c.before.erase(std::remove_if(c.before.begin(), c.before.end(), [&](size_t p) { return p > c.last; }), c.before.end());
  c.after.erase(std::remove_if(c.after.begin(), c.after.end(), [&](size_t p) { return p > c.last; }), c.after.end());
  auto roles = roles_of(plan, c);
  size_t reduces = (size_t)std::count(roles.begin(), roles.end(), Role::Reduce);
  size_t fulls = (size_t)std::count(roles.begin(), roles.end(), Role::Full);
  if (reduces == 0 || fulls == 0) return false;
  std::vector<size_t> outputs;
  for (auto& o : plan.outputs) outputs.push_back(o.slot);
  c.store.clear();
  size_t stored = 0, columns = 0;
  for (size_t m = 0; m < c.members.size(); ++m) {
    auto writes = step_writes(plan.steps[c.members[m]]);
    std::vector<bool> flags;
    for (size_t x : writes) {
      if (roles[m] != Role::Full) ++columns;
      bool later = false;
      for (size_t m2 = m + 1; m2 < c.members.size() && !later; ++m2) later = contains(step_writes(plan.steps[c.members[m2]]), x);
      for (size_t a : c.after) later = later || (a > c.members[m] && contains(step_writes(plan.steps[a]), x));
      bool live = false;
      if (!later) {
        live = contains(outputs, x);
        for (size_t q = c.last + 1; q < plan.steps.size(); ++q) {
          if (contains(step_reads(plan.steps[q]), x)) {
            live = true;
            break;
          }
          if (contains(step_writes(plan.steps[q]), x)) break;
        }
      }
      flags.push_back(live);
      stored += live;
    }
    c.store.push_back(flags);
  }
  std::vector<size_t> read_slots;
  for (size_t m = 0; m < c.members.size(); ++m)
    for (auto& in : row_inputs(plan, c, m))
      if (in.kind != RowInput::Value && !contains(read_slots, in.slot)) read_slots.push_back(in.slot);
  if (read_slots.size() > MAX_BINDINGS || stored > MAX_BINDINGS || columns > MAX_COLUMNS) return false;
  return buffers_needed(plan, c) <= MAX_BUFFERS;
}

bool try_chain(const Plan& plan, size_t start, RowChain* out) {
  const Step& s0 = plan.steps[start];
  std::vector<size_t> S;
  DType dt;
  if (s0.fused) {
    S = s0.group.shape;
    dt = s0.group.dtype;
  } else if (elementwise(s0.instr)) {
    S = s0.instr.shape;
    dt = s0.instr.dtype;
  } else if (s0.instr.op.kind == OpKind::Reduce && s0.instr.args.size() == 1) {
    S = s0.instr.arg_shapes[0];
    dt = s0.instr.dtype;
  } else {
    return false;
  }
  if (dt != DType::F32 && dt != DType::F64) return false;
  if (S.empty() || S.back() < 2) return false;
  const size_t cols = S.back(), rows = product(S) / cols;
  if (cols > (dt == DType::F32 ? MAX_COLS_F32 : MAX_COLS_F64) || rows * cols >= (size_t(1) << 31) || rows == 0) return false;
  Builder b(plan, S, dt);
  Role r0 = role_of(s0, b.S, b.dt);
  if (r0 != Role::Full && r0 != Role::Reduce) return false;
  b.c.shape = b.S;
  b.c.rows = rows;
  b.c.cols = cols;
  b.c.dtype = b.dt;
  size_t idle = 0;
  for (size_t p = start; p < plan.steps.size() && idle <= LOOKAHEAD; ++p) {
    if (b.try_member(p)) {
      idle = 0;
      continue;
    }
    if (b.c.members.empty()) return false;
    ++idle;
    if (!b.try_before(p) && !b.try_after(p)) break;
  }
  // Drop members from the end until the chain fits (a chain must end with what it can hold).
  RowChain c = b.c;
  while (!c.members.empty()) {
    RowChain t = c;
    if (finish(plan, t)) {
      *out = t;
      return true;
    }
    c.members.pop_back();
  }
  return false;
}

}  // namespace

std::vector<RowInput> row_inputs(const Plan& plan, const RowChain& c, size_t m) {
  Builder b(plan, c.shape, c.dtype);
  std::vector<RowInput> ins;
  for (size_t k = 0; k <= m; ++k) {
    size_t p = c.members[k];
    Role r = role_of(plan.steps[p], c.shape, c.dtype);
    ins.clear();
    b.classify(p, r, &ins);
    b.roles.push_back(r);
    auto writes = step_writes(plan.steps[p]);
    for (size_t q = 0; q < writes.size(); ++q) b.latest[writes[q]] = {k, q};
  }
  return ins;
}

std::vector<RowChain> find_row_chains(const Plan& plan, bool device_plan) {
  std::vector<RowChain> out;
  // Only plans built with the CUDA device's fusion configuration (the one with `sink`).
  if (!row_chains_enabled() || !(device_plan || plan.fuse.sink)) return out;
  size_t p = 0;
  while (p < plan.steps.size()) {
    RowChain c;
    if (try_chain(plan, p, &c)) {
      out.push_back(c);
      p = c.last + 1;
    } else {
      ++p;
    }
  }
  return out;
}

}  // namespace rg
