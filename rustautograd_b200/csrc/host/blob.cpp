// Plan serialisation for the C ABI.
#include "blob.h"

#include <cstring>
#include <stdexcept>

namespace rg {

namespace {

struct Writer {
  std::vector<uint8_t> out;
  void u8(uint8_t v) { out.push_back(v); }
  void u32(uint32_t v) { raw(&v, 4); }
  void u64(uint64_t v) { raw(&v, 8); }
  void raw(const void* p, size_t n) {
    const uint8_t* b = (const uint8_t*)p;
    out.insert(out.end(), b, b + n);
  }
  void vec(const std::vector<size_t>& v) {
    u64(v.size());
    for (size_t x : v) u64(x);
  }
  void tensor(const Tensor& t) {
    u8((uint8_t)t.dtype());
    vec(t.shape);
    u64(t.data.bytes());
    raw(t.data.data(), t.data.bytes());
  }
  void op(const Op& o) {
    u8((uint8_t)o.kind);
    u64(o.index);
    vec(o.shape);
    vec(o.starts);
    vec(o.stops);
    u8((uint8_t)o.dtype);
    u8(o.flag_a);
    u8(o.flag_b);
    u8((uint8_t)o.reduce);
    u8(o.value ? 1 : 0);
    if (o.value) tensor(*o.value);
    u64(o.n_carry);
    u64(o.n_x);
    u64(o.length);
    u64(o.max_iterations);
  }
  void plan(const Plan& p) {
    u64(p.slots.size());
    for (auto& [d, n] : p.slots) {
      u8((uint8_t)d);
      u64(n);
    }
    for (bool b : p.pinned) u8(b);
    u64(p.consts.size());
    for (auto& [s, t] : p.consts) {
      u64(s);
      tensor(*t);
    }
    u64(p.input_slots.size());
    for (size_t k = 0; k < p.input_slots.size(); ++k) {
      u64(p.input_slots[k]);
      u64(p.input_ns[k]);
    }
    u64(p.outputs.size());
    for (auto& o : p.outputs) {
      u64(o.slot);
      vec(o.shape);
      u64(o.n);
    }
    u8(p.reference);
    u64(p.naive_bytes);
    u64(p.peak_live_bytes);
    u64(p.steps.size());
    for (auto& st : p.steps) {
      u8(st.fused);
      if (st.fused) {
        const Fused& f = st.group;
        u8((uint8_t)f.dtype);
        u64(f.n);
        u64(f.inputs.size());
        for (auto& in : f.inputs) {
          u64(in.slot);
          u8((uint8_t)in.kind);
          u64(in.row);
          u64(in.reg);
        }
        u64(f.ops.size());
        for (auto& m : f.ops) {
          op(m.op);
          u64(m.reg);
          u64(m.args.size());
          for (auto& a : m.args) {
            u8(a.reg);
            u64(a.idx);
          }
        }
        u64(f.outputs.size());
        for (auto& [r, s] : f.outputs) {
          u64(r);
          u64(s);
        }
        u64(f.regs);
        vec(f.shape);
        u64(f.input_shapes.size());
        for (auto& s : f.input_shapes) vec(s);
      } else {
        const Instr& i = st.instr;
        op(i.op);
        u32(i.node);
        u8((uint8_t)i.dtype);
        u64(i.dst);
        vec(i.args);
        vec(i.shape);
        u64(i.arg_shapes.size());
        for (auto& s : i.arg_shapes) vec(s);
        u64(i.n);
        u8((uint8_t)i.mode);
        u64(i.outs.size());
        for (auto& [a, b] : i.outs) {
          u64(a);
          u64(b);
        }
        u8(i.body_plan ? 1 : 0);
        if (i.body_plan) plan(*i.body_plan);
        u8(i.body2_plan ? 1 : 0);
        if (i.body2_plan) plan(*i.body2_plan);
      }
    }
  }
};

struct Reader {
  const uint8_t* p;
  size_t n, at = 0;
  void need(size_t k) {
    if (at + k > n) throw std::runtime_error("plan blob truncated");
  }
  uint8_t u8() {
    need(1);
    return p[at++];
  }
  uint32_t u32() {
    uint32_t v;
    need(4);
    std::memcpy(&v, p + at, 4);
    at += 4;
    return v;
  }
  uint64_t u64() {
    uint64_t v;
    need(8);
    std::memcpy(&v, p + at, 8);
    at += 8;
    return v;
  }
  size_t count() {
    uint64_t c = u64();
    if (c > n) throw std::runtime_error("plan blob count out of range");
    return (size_t)c;
  }
  std::vector<size_t> vec() {
    size_t k = count();
    std::vector<size_t> v(k);
    for (auto& x : v) x = u64();
    return v;
  }
  DType dtype() {
    uint8_t d = u8();
    if (d > 2) throw std::runtime_error("plan blob has an unknown dtype");
    return (DType)d;
  }
  TensorP tensor() {
    DType d = dtype();
    auto shape = vec();
    size_t bytes = count();
    need(bytes);
    Buf b(d, product(shape));
    if (b.bytes() != bytes) throw std::runtime_error("plan blob tensor size mismatch");
    std::memcpy(b.data(), p + at, bytes);
    at += bytes;
    return std::make_shared<const Tensor>(shape, std::move(b));
  }
  Op op() {
    Op o;
    uint8_t k = u8();
    if (k > (uint8_t)OpKind::AttnBwd) throw std::runtime_error("plan blob has an unknown op");
    o.kind = (OpKind)k;
    o.index = u64();
    o.shape = vec();
    o.starts = vec();
    o.stops = vec();
    o.dtype = dtype();
    o.flag_a = u8();
    o.flag_b = u8();
    o.reduce = (ReduceKind)u8();
    if (u8()) o.value = tensor();
    o.n_carry = u64();
    o.n_x = u64();
    o.length = u64();
    o.max_iterations = u64();
    return o;
  }
  Plan plan() {
    Plan pl;
    size_t ns = count();
    for (size_t k = 0; k < ns; ++k) {
      DType d = dtype();
      pl.slots.emplace_back(d, (size_t)u64());
    }
    for (size_t k = 0; k < ns; ++k) pl.pinned.push_back(u8() != 0);
    size_t nc = count();
    for (size_t k = 0; k < nc; ++k) {
      size_t s = u64();
      pl.consts.emplace_back(s, tensor());
    }
    size_t ni = count();
    for (size_t k = 0; k < ni; ++k) {
      pl.input_slots.push_back(u64());
      pl.input_ns.push_back(u64());
    }
    size_t no = count();
    for (size_t k = 0; k < no; ++k) {
      PlanOutput o;
      o.slot = u64();
      o.shape = vec();
      o.n = u64();
      pl.outputs.push_back(o);
    }
    pl.reference = u8();
    pl.naive_bytes = u64();
    pl.peak_live_bytes = u64();
    size_t nst = count();
    for (size_t k = 0; k < nst; ++k) {
      Step st;
      st.fused = u8();
      if (st.fused) {
        Fused& f = st.group;
        f.dtype = dtype();
        f.n = u64();
        size_t nin = count();
        for (size_t j = 0; j < nin; ++j) {
          FusedInput in;
          in.slot = u64();
          in.kind = (ArgKind)u8();
          in.row = u64();
          in.reg = u64();
          f.inputs.push_back(in);
        }
        size_t nops = count();
        for (size_t j = 0; j < nops; ++j) {
          MicroOp m;
          m.op = op();
          m.reg = u64();
          size_t na = count();
          for (size_t a = 0; a < na; ++a) {
            Operand o;
            o.reg = u8();
            o.idx = u64();
            m.args.push_back(o);
          }
          f.ops.push_back(std::move(m));
        }
        size_t nout = count();
        for (size_t j = 0; j < nout; ++j) {
          size_t r = u64();
          f.outputs.emplace_back(r, (size_t)u64());
        }
        f.regs = u64();
        f.shape = vec();
        size_t nis = count();
        for (size_t j = 0; j < nis; ++j) f.input_shapes.push_back(vec());
      } else {
        Instr& i = st.instr;
        i.op = op();
        i.node = u32();
        i.dtype = dtype();
        i.dst = u64();
        i.args = vec();
        i.shape = vec();
        size_t nas = count();
        for (size_t j = 0; j < nas; ++j) i.arg_shapes.push_back(vec());
        i.n = u64();
        i.mode = (Mode)u8();
        size_t nouts = count();
        for (size_t j = 0; j < nouts; ++j) {
          size_t a = u64();
          i.outs.emplace_back(a, (size_t)u64());
        }
        if (u8()) i.body_plan = std::make_shared<Plan>(plan());
        if (u8()) i.body2_plan = std::make_shared<Plan>(plan());
      }
      pl.steps.push_back(std::move(st));
    }
    return pl;
  }
};

}  // namespace

std::vector<uint8_t> encode_plan(const Plan& p) {
  Writer w;
  w.raw("RGPL", 4);
  w.u32(PLAN_BLOB_VERSION);
  w.plan(p);
  return std::move(w.out);
}

Plan decode_plan(const uint8_t* data, size_t len) {
  Reader r{data, len};
  r.need(8);
  if (std::memcmp(data, "RGPL", 4) != 0) throw std::runtime_error("not a plan blob");
  r.at = 4;
  if (r.u32() != PLAN_BLOB_VERSION) throw std::runtime_error("unsupported plan blob version");
  Plan p = r.plan();
  if (r.at != len) throw std::runtime_error("trailing bytes after plan blob");
  // Validate slot references so a malformed blob is rejected here, not on the device.
  auto check = [&](const Plan& pl, auto&& self) -> void {
    size_t S = pl.slots.size();
    auto ok = [&](size_t s) {
      if (s >= S) throw std::runtime_error("plan blob references a slot out of range");
    };
    for (auto& c : pl.consts) {
      ok(c.first);
      if (c.second->n() > pl.slots[c.first].second) throw std::runtime_error("constant larger than its slot");
    }
    for (size_t k = 0; k < pl.input_slots.size(); ++k) {
      ok(pl.input_slots[k]);
      if (pl.input_ns[k] > pl.slots[pl.input_slots[k]].second) throw std::runtime_error("input larger than its slot");
    }
    for (auto& o : pl.outputs) {
      ok(o.slot);
      if (o.n > pl.slots[o.slot].second) throw std::runtime_error("output larger than its slot");
    }
    for (auto& st : pl.steps) {
      if (st.fused) {
        for (auto& in : st.group.inputs) ok(in.slot);
        for (auto& o : st.group.outputs) {
          ok(o.second);
          if (pl.slots[o.second].second < st.group.n) throw std::runtime_error("fused output slot too small");
        }
      } else {
        for (size_t a : st.instr.args) ok(a);
        if (!st.instr.op.is_control_flow()) {
          ok(st.instr.dst);
          if (pl.slots[st.instr.dst].second < st.instr.n) throw std::runtime_error("destination slot too small");
        }
        for (auto& o : st.instr.outs) ok(o.second);
        if (st.instr.body_plan) self(*st.instr.body_plan, self);
        if (st.instr.body2_plan) self(*st.instr.body2_plan, self);
      }
    }
  };
  check(p, check);
  return p;
}

}  // namespace rg
