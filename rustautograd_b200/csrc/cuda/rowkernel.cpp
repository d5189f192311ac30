// Row chains as generated kernels (rowkernel.h).
#include "rowkernel.h"

#include <algorithm>
#include <cstdio>
#include <functional>
#include <map>
#include <sstream>
#include <tuple>

namespace rgc {

using rg::DType;
using rg::OpKind;
using rg::RowInput;

namespace {

// Shared memory a block may use. The kernels are bound by memory latency as much as by
// bandwidth: a stage issues its loads, and the block then waits at a barrier before its
// reductions, so the SM needs several blocks in flight to keep HBM busy. About 44 KB per block
// lets five blocks (40 warps) share an SM; rows per block are capped so that each block still
// turns over often enough to overlap with the others.
constexpr size_t SMEM_TARGET = 44 * 1024, SMEM_MAX = 200 * 1024;
constexpr int MAX_ROWS_PER_BLOCK = 32;

enum class Role { Full, Col, Reduce };

struct Member {
  Role role = Role::Full;
  int stage = 0;
  ElemSpec spec;                 // elementwise members
  std::vector<int> in_reg;       // spec input -> register (non-full spec inputs), else -1
  std::vector<RowInput> ins;
  std::vector<size_t> writes;    // output slots
  rg::ReduceKind red = rg::ReduceKind::Sum;
};

struct Val {
  int buf = -1;  // full value kept in shared memory for later stages
  int col = -1;  // per-row value (always kept)
  int out = -1;  // ElemArgs::out index when stored
};

struct Bind {
  RowInput in;
  bool full_reader = true;  // read by full or reduction members (else by per-row members)
  int buf = -1;             // kept in shared memory (read by a reduction or in several stages)
  int loaded = -1;          // stage that loads it into `buf`
  int bc = -1;
  std::vector<int> stages;
};

std::string L(long long v) { return std::to_string(v) + "LL"; }
std::string I(long long v) { return std::to_string(v); }
const char* lane(int j) {
  static const char* n[] = {"x", "y", "z", "w"};
  return n[j];
}

}  // namespace

bool make_row_kernel(const rg::Plan& plan, const rg::RowChain& c, RowKernel* k, std::string* why) {
  const DType dt = c.dtype;
  const std::string T = elem_ctype(dt), VT = dt == DType::F64 ? "double2" : "float4";
  const long long C = (long long)c.cols, R = (long long)c.rows;
  const size_t esz = rg::dtype_size(dt);
  const int G = dt == DType::F32 ? (C % 4 == 0 ? 4 : 1) : (C % 2 == 0 ? 2 : 1);
  const long long CV = C / G;
  std::vector<size_t> S = c.shape, Sc = c.shape;
  Sc.back() = 1;
  *k = RowKernel();

  // Members, their stages and inputs.
  std::vector<Member> ms;
  int stage = -1;
  Role prev = Role::Full;
  for (size_t m = 0; m < c.members.size(); ++m) {
    const rg::Step& st = plan.steps[c.members[m]];
    Member mb;
    const auto& shape = st.fused ? st.group.shape : st.instr.shape;
    if (!st.fused && st.instr.op.kind == OpKind::Reduce) {
      mb.role = Role::Reduce;
      mb.red = st.instr.op.reduce;
    } else {
      mb.role = shape == S ? Role::Full : Role::Col;
      mb.spec = st.fused ? spec_from_group(st.group) : spec_from_instr(st.instr);
      int r = 0;
      for (auto& in : mb.spec.inputs) mb.in_reg.push_back(in.kind == rg::ArgKind::Full ? -1 : r++);
    }
    if (m == 0 || mb.role != prev || mb.role == Role::Reduce) ++stage;
    prev = mb.role;
    mb.stage = stage;
    mb.ins = rg::row_inputs(plan, c, m);
    mb.writes = rg::step_writes(st);
    if (mb.role != Role::Reduce && mb.ins.size() != mb.spec.inputs.size()) {
      *why = "member inputs do not match its kernel inputs";
      return false;
    }
    ms.push_back(std::move(mb));
  }
  const int stages = stage + 1;

  // Values: full ones read in a later stage get a shared-memory buffer, per-row ones an array.
  std::map<std::pair<size_t, size_t>, Val> vals;
  int nbuf = 0, ncol = 0;
  for (size_t m = 0; m < ms.size(); ++m)
    for (auto& in : ms[m].ins)
      if (in.kind == RowInput::Value && ms[in.producer].role == Role::Full && ms[in.producer].stage != ms[m].stage) {
        Val& v = vals[{in.producer, in.output}];
        if (v.buf < 0) v.buf = nbuf++;
      }
  for (size_t m = 0; m < ms.size(); ++m)
    if (ms[m].role != Role::Full)
      for (size_t q = 0; q < ms[m].writes.size(); ++q) vals[{m, q}].col = ncol++;
  for (size_t m = 0; m < ms.size(); ++m)
    for (size_t q = 0; q < ms[m].writes.size(); ++q)
      if (c.store[m][q]) {
        vals[{m, q}].out = (int)k->out_slots.size();
        k->out_slots.push_back(ms[m].writes[q]);
      }

  // Slots read from outside the chain, one kernel parameter each per way of reading.
  std::vector<Bind> binds;
  std::map<std::tuple<int, size_t, size_t, std::vector<size_t>, bool>, int> bind_of;
  std::vector<std::vector<int>> member_bind(ms.size());
  for (size_t m = 0; m < ms.size(); ++m) {
    for (auto& in : ms[m].ins) {
      if (in.kind == RowInput::Value) {
        member_bind[m].push_back(-1);
        continue;
      }
      bool full_reader = ms[m].role != Role::Col;
      auto key = std::make_tuple((int)in.kind, in.slot, in.period, in.shape, full_reader);
      auto it = bind_of.find(key);
      int b;
      if (it == bind_of.end()) {
        b = (int)binds.size();
        Bind nb;
        nb.in = in;
        nb.full_reader = full_reader;
        binds.push_back(nb);
        bind_of[key] = b;
      } else {
        b = it->second;
      }
      binds[b].stages.push_back(ms[m].stage);
      if (ms[m].role == Role::Reduce) binds[b].stages.push_back(-1 - ms[m].stage);  // marks a reduction reader
      member_bind[m].push_back(b);
    }
  }
  for (auto& b : binds) {
    if (b.in.kind != RowInput::Full || !b.full_reader) continue;
    bool reduced = false, several = false;
    for (int s : b.stages) {
      if (s < 0) reduced = true;
      else if (s != b.stages[0]) several = true;
    }
    if (reduced || several) b.buf = nbuf++;
  }
  for (size_t q = 0; q < binds.size(); ++q) {
    Bind& b = binds[q];
    FDiv div{};
    if (b.in.kind == RowInput::Periodic) div = make_fdiv(b.in.period);
    if (b.in.kind == RowInput::Broadcast || b.in.kind == RowInput::Source) {
      const auto& shape = b.full_reader ? S : Sc;
      auto st = rg::bstrides(b.in.shape, shape.size());
      Dims d;
      if (shape.size() > (size_t)MAXR) {
        *why = "rank above 8";
        return false;
      }
      d.rank = (int)shape.size();
      for (size_t x = 0; x < shape.size(); ++x) {
        d.d[x] = (long long)shape[x];
        d.st[x] = (long long)st[x];
      }
      bool ok = false;
      FDims f = fast_dims(d, &ok);
      if (!ok) {
        *why = "a broadcast extent does not fit 32-bit index math";
        return false;
      }
      b.bc = (int)k->bcs.size();
      k->bcs.push_back(f);
    }
    k->in_slots.push_back(b.in.slot);
    k->in_div.push_back(div);
  }
  if (binds.size() > (size_t)JIT_MAX_IN || k->out_slots.size() > (size_t)JIT_MAX_OUT) {
    *why = "too many operands";
    return false;
  }

  // Geometry: a row pitch of 8 (mod 32) 4-byte words, so that the eight lanes summing each of
  // four rows of a warp meet no bank twice, and a multiple of the vector width.
  long long pitch = C;
  while (((pitch * (long long)esz / 4) % 32) != 8 || pitch % G != 0) ++pitch;
  const size_t row_bytes = ((size_t)nbuf * (size_t)pitch + (size_t)ncol) * esz;
  int rb = row_bytes ? (int)std::min<size_t>(MAX_ROWS_PER_BLOCK, SMEM_TARGET / row_bytes) : MAX_ROWS_PER_BLOCK;
  rb = rb / 4 * 4;
  if (rb < 4) {
    rb = 4;
    if (4 * row_bytes > SMEM_MAX) {
      *why = "a block of rows does not fit shared memory";
      return false;
    }
  }
  while (rb > 4 && rb - 4 >= R) rb -= 4;
  const long long RB = rb, P = pitch;
  k->rows = R;
  k->rows_per_block = rb;
  k->smem = (size_t)rb * row_bytes;

  // ---- source ----
  std::ostringstream o;
  auto in_ptr = [&](int b) { return "((const " + T + "*)a.in[" + I(b) + "])"; };
  auto out_ptr = [&](int q) { return "((" + T + "*)a.out[" + I(q) + "])"; };
  auto fbuf = [&](int buf) { return "(F + " + L(buf * RB * P) + ")"; };
  auto kcol = [&](int col) { return "K[" + I(col * RB) + " + rl]"; };
  o << "(const ElemArgs a) {\n";
  o << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
  o << "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
  o << "  extern __shared__ __align__(16) unsigned char rg_smem[];\n";
  o << "  " << T << "* const F = (" << T << "*)rg_smem;\n";
  o << "  " << T << "* const K = F + " << L((long long)nbuf * RB * P) << ";\n";
  for (size_t b = 0; b < binds.size(); ++b)
    if (binds[b].in.kind == RowInput::Splat) o << "  const " << T << " sp" << b << " = " << in_ptr((int)b) << "[0];\n";
  o << "  const long long R = a.n;\n";
  o << "  for (long long r0 = (long long)blockIdx.x * " << L(RB) << "; r0 < R; r0 += (long long)gridDim.x * " << L(RB) << ") {\n";
  o << "    const int nr = (int)(R - r0 < " << L(RB) << " ? R - r0 : " << L(RB) << ");\n";

  // Loads binding b into x<b>[0..W) for the element(s) at e (full space) or row e (per-row space).
  auto load_bind = [&](int b, int W, int st_now, bool full_space) {
    Bind& bd = binds[b];
    std::string x = "x" + I(b);
    o << "      " << T << " " << x << "[" << W << "];\n";
    switch (bd.in.kind) {
      case RowInput::Full:
        if (full_space && bd.buf >= 0 && bd.loaded >= 0 && bd.loaded < st_now) {
          o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << x << "[q] = " << fbuf(bd.buf) << "[rl * " << P << " + j + q];\n";
        } else if (full_space && W > 1) {
          o << "      { const " << VT << " w = *(const " << VT << "*)(" << in_ptr(b) << " + e);";
          for (int j = 0; j < W; ++j) o << " " << x << "[" << j << "] = w." << lane(j) << ";";
          o << " }\n";
          if (bd.buf >= 0 && (bd.loaded < 0 || bd.loaded == st_now)) {
            o << "      { " << VT << " w;";
            for (int j = 0; j < W; ++j) o << " w." << lane(j) << " = " << x << "[" << j << "];";
            o << " *(" << VT << "*)(" << fbuf(bd.buf) << " + rl * " << P << " + j) = w; }\n";
            bd.loaded = st_now;
          }
        } else {
          o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << x << "[q] = " << in_ptr(b) << "[e + q];\n";
          if (full_space && bd.buf >= 0 && (bd.loaded < 0 || bd.loaded == st_now)) {
            o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << fbuf(bd.buf) << "[rl * " << P << " + j + q] = " << x << "[q];\n";
            bd.loaded = st_now;
          }
        }
        break;
      case RowInput::Column:
        o << "      { const " << T << " v = " << in_ptr(b) << "[r0 + rl];\n      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << x
          << "[q] = v; }\n";
        break;
      case RowInput::Splat:
        o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << x << "[q] = sp" << b << ";\n";
        break;
      case RowInput::Periodic:
        o << "      rg_row_fill<" << T << ", " << W << ">(" << x << ", " << in_ptr(b) << ", e, a.row[" << b << "]);\n";
        break;
      default:
        o << "      rg_bc_fill<" << T << ", " << W << ">(" << x << ", " << in_ptr(b) << ", a.bc[" << bd.bc << "], e);\n";
        break;
    }
  };

  // The elementwise members of stage `s` over W lanes.
  auto members_code = [&](int s, int W) {
    for (size_t m = 0; m < ms.size(); ++m) {
      if (ms[m].stage != s) continue;
      const Member& mb = ms[m];
      std::string P0 = "m" + I((long long)m) + "_";
      for (size_t q = 0; q < mb.ins.size(); ++q) {
        const RowInput& in = mb.ins[q];
        std::string dst = mb.in_reg[q] < 0 ? P0 + "i" + I((long long)q) : P0 + "r" + I(mb.in_reg[q]);
        std::string src;
        if (in.kind != RowInput::Value) {
          src = "x" + I(member_bind[m][q]) + "[q]";
        } else {
          const Member& pm = ms[in.producer];
          const Val& v = vals[{in.producer, in.output}];
          if (pm.role != Role::Full) {
            src = pm.stage == s ? "m" + I((long long)in.producer) + "_r" + I((long long)pm.spec.out_regs[in.output]) + "[q]" : kcol(v.col);
          } else if (pm.stage == s) {
            src = "m" + I((long long)in.producer) + "_r" + I((long long)pm.spec.out_regs[in.output]) + "[q]";
          } else {
            src = fbuf(v.buf) + "[rl * " + I(P) + " + j + q]";
          }
        }
        o << "      " << T << " " << dst << "[" << W << "];\n";
        o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << dst << "[q] = " << src << ";\n";
      }
      for (auto& op : mb.spec.ops) {
        std::vector<std::string> args;
        for (auto& x : op.args) args.push_back(P0 + (x.reg ? "r" : "i") + I((long long)x.idx) + "[q]");
        o << "      " << T << " " << P0 << "r" << op.reg << "[" << W << "];\n";
        o << "      #pragma unroll\n      for (int q = 0; q < " << W << "; ++q) " << P0 << "r" << op.reg << "[q] = " << elem_expr(dt, op.op, args)
          << ";\n";
      }
    }
  };

  for (int s = 0; s < stages; ++s) {
    Role role = Role::Full;
    for (auto& mb : ms)
      if (mb.stage == s) role = mb.role;
    std::vector<int> used;
    for (size_t m = 0; m < ms.size(); ++m)
      if (ms[m].stage == s)
        for (int b : member_bind[m])
          if (b >= 0 && std::find(used.begin(), used.end(), b) == used.end()) used.push_back(b);
    o << "    // stage " << s << "\n";
    if (role == Role::Full) {
      // Unrolled, so that the loads of several iterations can be in flight together where the
      // compiler can order them ahead of the earlier iterations' stores.
      o << "    #pragma unroll 4\n";
      o << "    for (int v = threadIdx.x; v < nr * " << CV << "; v += " << ROW_THREADS << ") {\n";
      o << "      const int rl = v / " << CV << ", j = (v - rl * " << CV << ") * " << G << ";\n";
      o << "      const unsigned e = (unsigned)((r0 + rl) * " << L(C) << " + j);\n";
      for (int b : used) load_bind(b, G, s, true);
      members_code(s, G);
      for (size_t m = 0; m < ms.size(); ++m) {
        if (ms[m].stage != s) continue;
        for (size_t q = 0; q < ms[m].writes.size(); ++q) {
          const Val& v = vals[{m, q}];
          std::string r = "m" + I((long long)m) + "_r" + I((long long)ms[m].spec.out_regs[q]);
          if (v.buf >= 0) {
            if (G > 1) {
              o << "      { " << VT << " w;";
              for (int j = 0; j < G; ++j) o << " w." << lane(j) << " = " << r << "[" << j << "];";
              o << " *(" << VT << "*)(" << fbuf(v.buf) << " + rl * " << P << " + j) = w; }\n";
            } else {
              o << "      " << fbuf(v.buf) << "[rl * " << P << " + j] = " << r << "[0];\n";
            }
          }
          if (v.out >= 0) {
            if (G > 1) {
              o << "      { " << VT << " w;";
              for (int j = 0; j < G; ++j) o << " w." << lane(j) << " = " << r << "[" << j << "];";
              o << " *(" << VT << "*)(" << out_ptr(v.out) << " + e) = w; }\n";
            } else {
              o << "      " << out_ptr(v.out) << "[e] = " << r << "[0];\n";
            }
          }
        }
      }
      o << "    }\n";
    } else if (role == Role::Col) {
      o << "    for (int rl = threadIdx.x; rl < nr; rl += " << ROW_THREADS << ") {\n";
      o << "      const unsigned e = (unsigned)(r0 + rl);\n      (void)e;\n";
      for (int b : used) load_bind(b, 1, s, false);
      members_code(s, 1);
      for (size_t m = 0; m < ms.size(); ++m) {
        if (ms[m].stage != s) continue;
        for (size_t q = 0; q < ms[m].writes.size(); ++q) {
          const Val& v = vals[{m, q}];
          std::string r = "m" + I((long long)m) + "_r" + I((long long)ms[m].spec.out_regs[q]) + "[0]";
          o << "      " << kcol(v.col) << " = " << r << ";\n";
          if (v.out >= 0) o << "      " << out_ptr(v.out) << "[e] = " << r << ";\n";
        }
      }
      o << "    }\n";
    } else {
      size_t m = 0;
      while (ms[m].stage != s) ++m;
      const Member& mb = ms[m];
      const RowInput& in = mb.ins[0];
      std::string row_base;
      if (in.kind == RowInput::Value) {
        row_base = fbuf(vals[{in.producer, in.output}].buf);
      } else {
        Bind& bd = binds[member_bind[m][0]];
        if (bd.loaded < 0) {
          // First read by this reduction: copy the block's rows into shared memory.
          o << "    for (int v = threadIdx.x; v < nr * " << C << "; v += " << ROW_THREADS << ") {\n";
          o << "      const int rl = v / " << C << ", j = v - rl * " << C << ";\n";
          o << "      " << fbuf(bd.buf) << "[rl * " << P << " + j] = " << in_ptr(member_bind[m][0]) << "[(r0 + rl) * " << L(C) << " + j];\n";
          o << "    }\n    __syncthreads();\n";
          bd.loaded = s;
        }
        row_base = fbuf(bd.buf);
      }
      const Val& v = vals[{m, 0}];
      const long long C8 = C / 8 * 8;
      o << "    {\n";
      o << "      const int lane = threadIdx.x & 31, sub = lane >> 3, k8 = lane & 7;\n";
      o << "      for (int base = (threadIdx.x >> 5) * 4; base < " << RB << "; base += " << ROW_THREADS / 8 << ") {\n";
      o << "        const int rl = base + sub;\n        const bool ok = rl < nr;\n";
      o << "        const " << T << "* row = " << row_base << " + (ok ? rl : 0) * " << P << ";\n";
      if (mb.red == rg::ReduceKind::Sum) {
        o << "        " << T << " acc = (" << T << ")0;\n";
        o << "        if (ok)\n          for (int c = k8; c < " << C8 << "; c += 8) acc = acc + row[c];\n";
        o << "        " << T << " out = (" << T << ")0;\n";
        o << "        #pragma unroll\n        for (int q = 0; q < 8; ++q) out = out + __shfl_sync(0xffffffffu, acc, (sub << 3) + q);\n";
        o << "        if (ok && k8 == 0) {\n";
        if (C8 < C) o << "          for (int c = " << C8 << "; c < " << C << "; ++c) out = out + row[c];\n";
      } else {
        const bool mx = mb.red == rg::ReduceKind::Max;
        const std::string gt = mx ? ">" : "<", ge = mx ? ">=" : "<=";
        const std::string inf = dt == DType::F64 ? "__longlong_as_double(0x7ff0000000000000LL)" : "__int_as_float(0x7f800000)";
        o << "        " << T << " acc = " << (mx ? "-" : "") << inf << ";\n        int idx = -1;\n";
        o << "        if (ok)\n          for (int c = k8; c < " << C << "; c += 8) {\n";
        o << "            const " << T << " x = row[c];\n";
        o << "            if (!(acc " << gt << " x) && x " << ge << " acc) idx = c;\n";
        o << "            acc = " << (mx ? "rg_max" : "rg_min") << "<" << T << ">(acc, x);\n          }\n";
        o << "        bool nan = false;\n        " << T << " out = acc;\n        int at = idx;\n";
        o << "        #pragma unroll\n        for (int q = 0; q < 8; ++q) {\n";
        o << "          const " << T << " y = __shfl_sync(0xffffffffu, acc, (sub << 3) + q);\n";
        o << "          const int yi = __shfl_sync(0xffffffffu, idx, (sub << 3) + q);\n";
        o << "          nan = nan || y != y;\n";
        o << "          if (yi >= 0 && (at < 0 || y " << gt << " out || (y == out && yi > at))) { out = y; at = yi; }\n";
        o << "        }\n";
        o << "        if (nan) out = rg_nan(out);\n";
        o << "        if (ok && k8 == 0) {\n";
      }
      o << "          " << kcol(v.col) << " = out;\n";
      if (v.out >= 0) o << "          " << out_ptr(v.out) << "[r0 + rl] = out;\n";
      o << "        }\n      }\n    }\n";
    }
    o << "    __syncthreads();\n";
  }
  o << "  }\n}\n";
  std::string body = o.str();
  char nm[64];
  snprintf(nm, sizeof nm, "rg_rows_%016llx", (unsigned long long)std::hash<std::string>{}(body + "rb" + I(RB)));
  k->name = nm;
  k->source = "extern \"C\" __global__ void __launch_bounds__(" + I(ROW_THREADS) + ") " + k->name + body;
  return true;
}

}  // namespace rgc
