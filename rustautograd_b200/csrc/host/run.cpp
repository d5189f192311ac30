// The generic multi-step loop and one-off execution over the Exec contract.
#include <algorithm>
#include <map>
#include <chrono>
#include <cmath>
#include <stdexcept>
#include <tuple>

#include "exec.h"
#include "rowchain.h"

namespace rg {

std::vector<Tensor> run_once(Device& d, const Plan& plan, const std::vector<const Tensor*>& inputs) {
  auto prog = d.compile(plan);
  auto e = prog->exec();
  for (size_t k = 0; k < inputs.size(); ++k) e->load(k, *inputs[k]);
  e->step();
  if (auto f = e->failure()) throw std::runtime_error("device execution failed: " + *f);
  std::vector<Tensor> out;
  for (auto& o : plan.outputs) out.emplace_back(o.shape, e->prefix(o.slot, o.n));
  return out;
}

// validate.rs:290-363. State moves by swapping buffers when the output's slot is private and of
// the same capacity, by copying otherwise; the run stops after the first step whose history
// scalars are not finite, with that step's state committed.
RunOut run_loop(const Plan& p, Exec& e, const RunSpec& spec, const std::vector<Tensor>& state,
                const std::vector<std::vector<Tensor>>& batches, size_t steps) {
  for (size_t k = 0; k < spec.state.size() && k < state.size(); ++k) e.load(spec.state[k].first, state[k]);
  auto load_batch = [&](const std::vector<Tensor>& b) {
    for (size_t k = 0; k < spec.data.size() && k < b.size(); ++k) e.load(spec.data[k], b[k]);
  };
  if (batches.size() == 1) load_batch(batches[0]);

  std::vector<size_t> out_slots;
  for (auto& io : spec.state) out_slots.push_back(p.outputs[io.second].slot);
  std::vector<std::pair<size_t, size_t>> swaps;
  std::vector<std::tuple<size_t, size_t, size_t>> copies;
  for (auto& io : spec.state) {
    size_t is = p.input_slots[io.first], os = p.outputs[io.second].slot;
    if (is == os) continue;
    size_t users = 0;
    for (size_t s : out_slots) users += s == os;
    if (!p.pinned[os] && users == 1 && p.slots[os].second == p.slots[is].second) swaps.emplace_back(is, os);
    else copies.emplace_back(is, os, p.outputs[io.second].n);
  }
  std::vector<size_t> hist_slots;
  for (size_t o : spec.history) hist_slots.push_back(p.outputs[o].slot);

  RunOut r;
  r.history.assign(hist_slots.size(), {});
  for (auto& h : r.history) h.reserve(steps);
  auto started = std::chrono::steady_clock::now();
  for (size_t k = 0; k < steps; ++k) {
    if (batches.size() > 1) load_batch(batches[k % batches.size()]);
    e.step();
    r.device_error = e.failure();
    if (r.device_error) break;
    r.steps = k + 1;
    bool bad = false;
    for (size_t h = 0; h < hist_slots.size(); ++h) {
      double v = e.scalar(hist_slots[h]);
      bad = bad || !std::isfinite(v);
      r.history[h].push_back(v);
    }
    if (bad) r.nonfinite_step = k;
    if (k + 1 == steps || bad) {
      r.outputs.clear();
      for (auto& o : p.outputs) r.outputs.emplace_back(o.shape, e.prefix(o.slot, o.n));
    }
    std::vector<std::pair<size_t, Buf>> temp;
    for (auto& c : copies) temp.emplace_back(std::get<0>(c), e.prefix(std::get<1>(c), std::get<2>(c)));
    for (auto& sw : swaps) e.swap(sw.first, sw.second);
    for (auto& t : temp) e.write_prefix(t.first, t.second);
    if (bad) break;
  }
  r.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - started).count();
  for (auto& io : spec.state)
    r.state.emplace_back(p.outputs[io.second].shape, e.prefix(p.input_slots[io.first], p.input_ns[io.first]));
  return r;
}

std::vector<StepCost> step_costs(const Plan& p) {
  std::vector<StepCost> out;
  for (auto& st : p.steps) {
    StepCost c;
    if (st.fused) {
      const Fused& f = st.group;
      c.kind = "fused";
      double es = (double)dtype_size(f.dtype);
      // Full inputs and outputs stream once; splats, rows and broadcasts are reused from cache.
      double full = 0;
      for (auto& in : f.inputs) full += in.kind == ArgKind::Full ? 1.0 : 0.0;
      c.bytes = (double)f.n * es * (full + (double)f.outputs.size());
      c.flops = (double)f.n * (double)f.ops.size();
      out.push_back(c);
      continue;
    }
    const Instr& i = st.instr;
    c.kind = i.op.name();
    double es = (double)dtype_size(i.dtype);
    double in_bytes = 0;
    for (size_t k = 0; k < i.arg_shapes.size(); ++k) in_bytes += (double)product(i.arg_shapes[k]) * es;
    if (i.op.kind == OpKind::MatMul || i.op.kind == OpKind::MatMulT) {
      c.kind = "matmul";
      const auto &sa = i.arg_shapes[0], &sb = i.arg_shapes[1];
      bool ta = i.op.kind == OpKind::MatMulT && i.op.flag_a;
      double k = sa.size() >= 2 ? (double)(ta ? sa[sa.size() - 2] : sa.back()) : (double)sa[0];
      (void)sb;
      c.flops = 2.0 * (double)i.n * k;
      c.bytes = in_bytes + (double)i.n * es;
    } else if (i.op.kind == OpKind::AttnFwd || i.op.kind == OpKind::AttnBwd) {
      // Products per batch entry: q k^T and P v forward; the backward recomputes q k^T and forms
      // dO v^T, P^T dO, dS k and dS^T q.
      const auto& q = i.arg_shapes[0];
      const bool packed = i.op.value && i.op.value->n() == 3;  // q, k, v as one (B, T, 3, H, d) tensor
      const double t = packed ? (double)q[1] : (double)q[q.size() - 2], d = (double)q.back();
      const double dv = packed ? d : (double)i.arg_shapes[2].back();
      const double batch = packed ? (double)(q[0] * q[3]) : (double)product(q) / (t * d);
      c.kind = "attention";
      c.flops = 2.0 * batch * t * t * (i.op.kind == OpKind::AttnFwd ? d + dv : 3.0 * d + 2.0 * dv);
      c.bytes = in_bytes + (double)i.n * es;
    } else if (i.op.kind == OpKind::Reduce) {
      c.flops = in_bytes / es;
      c.bytes = in_bytes + (double)i.n * es;
    } else {
      c.bytes = in_bytes + (double)i.n * es;
      c.flops = 0;
    }
    out.push_back(c);
  }
  // A row chain (on unless RGC_ROW_CHAINS=0) runs as one kernel at its first step: it reads each slot it
  // reads from outside once and writes only the values it stores. Its members' own costs give
  // way to that, so that time and bytes per step stay paired.
  for (auto& ch : find_row_chains(p)) {
    const double es = (double)dtype_size(ch.dtype), full = (double)ch.rows * (double)ch.cols, rows = (double)ch.rows;
    double bytes = 0, flops = 0;
    // Each slot read from outside counts once, at the largest extent any member reads it (one
    // member may read a slot in full where another reads one value per row of it).
    std::map<size_t, double> reads;
    for (size_t m = 0; m < ch.members.size(); ++m) {
      const Step& st = p.steps[ch.members[m]];
      // Per-row members read and write (..., 1) values; full ones and reductions read rows.
      const bool per_row = !(st.fused ? st.group.shape == ch.shape : (st.instr.shape == ch.shape || st.instr.op.kind == OpKind::Reduce));
      const bool full_out = st.fused ? st.group.shape == ch.shape : st.instr.shape == ch.shape;
      flops += out[ch.members[m]].flops;
      for (auto& in : row_inputs(p, ch, m)) {
        if (in.kind == RowInput::Value) continue;
        double b = 0;
        switch (in.kind) {
          case RowInput::Full: b = (per_row ? rows : full) * es; break;
          case RowInput::Column: b = rows * es; break;
          case RowInput::Periodic: b = (double)in.period * es; break;
          case RowInput::Splat: b = es; break;
          default: b = (double)product(in.shape) * es; break;
        }
        double& r = reads[in.slot];
        r = std::max(r, b);
      }
      auto writes = step_writes(st);
      for (size_t q = 0; q < writes.size(); ++q)
        if (ch.store[m][q]) bytes += (full_out ? full : rows) * es;
      out[ch.members[m]] = StepCost{"row_chain", 0.0, 0.0};
    }
    for (auto& [slot, b] : reads) bytes += b;
    out[ch.first] = StepCost{"row_chain", flops, bytes};
  }
  return out;
}

}  // namespace rg
