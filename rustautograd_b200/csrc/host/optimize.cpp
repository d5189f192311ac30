// Restates src/optimize.rs (line references below are to that file).
#include "optimize.h"

#include <cstring>

#include <algorithm>
#include <cstdlib>
#include <functional>
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
// the backward pass to bound the memory of a unified-memory GPU, choosing them by memory. The
// device instead recomputes what saves traffic (recompute_in_consumers below) and keeps every
// other activation while the plan peaks at no more than this share of its 180 GB of HBM (the
// rest holds the state snapshot, GEMM scratch and control-flow body frames). Above it rg's
// rematerialisation bounds memory, transcendental values included. Recomputation gives the same
// values, so results do not change.
constexpr size_t DEVICE_ACTIVATIONS_BYTES = size_t(120) << 30;

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

// The device's own rematerialisation (no counterpart in rg): an elementwise forward value that
// only elementwise consumers of its shape read is recomputed by its backward consumers when the
// values it derives from include at most one full-size tensor that is stored anyway (a product's
// output, a reduction's input, a value another kind of step reads). The clones run inside the
// backward group that reads them (adjacent to it in graph order, or moved to its level by
// Fuse::sink), so the forward group no longer writes the value and the backward group reads the
// stored source instead: the GELU of an MLP block then writes only its output, and its backward
// reads the product h = x W + b instead of six intermediates. Clones are the same operations
// on the same inputs, so every value is unchanged. rg's own rematerialisation (above) chooses
// what to recompute to bound memory and recomputes values that are stored anyway.
std::pair<Graph, std::vector<uint32_t>> recompute_in_consumers(const Graph& g, const std::vector<uint32_t>& outputs,
                                                               const std::vector<bool>& backward, OptStats& st) {
  const size_t N = g.nodes.size();
  auto keep = g.reachable(outputs);
  auto elementwise = [&](size_t i) {
    const Node& n = g.nodes[i];
    return keep[i] && !is_leaf(n) && n.dtype != DType::I32 &&
           (n.op.is_unary_elementwise() || n.op.is_binary_elementwise() || n.op.kind == OpKind::Where);
  };
  std::vector<std::vector<size_t>> users(N);
  for (size_t i = 0; i < N; ++i)
    if (keep[i] && !is_leaf(g.nodes[i]))
      for (auto x : g.nodes[i].inputs) users[x].push_back(i);
  std::vector<bool> output(N, false);
  for (auto o : outputs) output[o] = true;
  // Stored anyway: anything but an elementwise node, an output, or a value some step other than an
  // elementwise node of its shape and dtype reads.
  std::vector<bool> stored(N, false);
  for (size_t i = 0; i < N; ++i) {
    if (!keep[i]) continue;
    bool s = !elementwise(i) || output[i];
    for (size_t u : users[i])
      s = s || !elementwise(u) || g.nodes[u].shape != g.nodes[i].shape || g.nodes[u].dtype != g.nodes[i].dtype;
    stored[i] = s;
  }
  auto full = [&](size_t x, size_t like) { return g.nodes[x].shape == g.nodes[like].shape && g.nodes[x].n() >= REMAT_MIN; };
  // The forward values a recomputation of `i` goes through (`i` and its unstored elementwise
  // ancestors of its shape) and the full-size stored values it starts from.
  constexpr size_t MAX_CHAIN = 48;
  std::vector<bool> recompute(N, false);
  for (size_t i = 0; i < N; ++i) {
    if (!keep[i] || backward[i] || stored[i] || !elementwise(i) || !full(i, i)) continue;
    bool read_by_backward = false;
    for (size_t u : users[i]) read_by_backward = read_by_backward || backward[u];
    if (!read_by_backward) continue;
    std::vector<size_t> chain, todo{i}, sources;
    std::vector<bool> seen_here;
    bool ok = true;
    while (!todo.empty() && ok) {
      size_t v = todo.back();
      todo.pop_back();
      if (std::find(chain.begin(), chain.end(), v) != chain.end()) continue;
      chain.push_back(v);
      ok = chain.size() <= MAX_CHAIN;
      for (auto x : g.nodes[v].inputs) {
        bool through = !backward[x] && !stored[x] && elementwise(x) && full(x, i);
        if (through) todo.push_back(x);
        else if (full(x, i) && std::find(sources.begin(), sources.end(), (size_t)x) == sources.end()) sources.push_back(x);
      }
    }
    recompute[i] = ok && sources.size() <= 1;
  }
  // Every forward value a recomputed one goes through is recomputed with it.
  for (size_t i = N; i-- > 0;)
    if (recompute[i])
      for (auto x : g.nodes[i].inputs)
        if (!backward[x] && !stored[x] && elementwise(x) && full(x, i)) recompute[x] = true;
  Graph h;
  std::vector<uint32_t> map(N, UINT32_MAX);
  std::vector<int64_t> clone(N, -1);
  std::function<uint32_t(uint32_t)> value = [&](uint32_t i) -> uint32_t {
    if (!recompute[i]) return map[i];
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


// GPU planning: a slice of a constant is a constant, made at plan time. The causal mask of a
// GPT is `tril[:t, :t]`: as a plan step its output slot is free for reuse once the mask's
// broadcast has run, and the allocator hands it to a later step, so row chains must read the
// materialised (B, H, T, T) broadcast. As a constant it is pinned, and the chains read the
// (T, T) source through the broadcast, once per row period. The values are the slice's own.
// Only slices of at most 2^22 elements fold, so constants stay small.
std::optional<Tensor> slice_of_constant(const Graph& g, uint32_t src, const Op& op, const std::vector<size_t>& shape) {
  const Node& n = g.nodes[src];
  if (n.op.kind != OpKind::Const || !n.op.value || shape.empty() || product(shape) > (size_t(1) << 22)) return std::nullopt;
  const Tensor& t = *n.op.value;
  const size_t rank = t.shape.size(), es = dtype_size(t.dtype());
  if (op.starts.size() != rank || shape.size() != rank) return std::nullopt;
  std::vector<size_t> stride(rank, 1);
  for (size_t k = rank; k-- > 1;) stride[k - 1] = stride[k] * t.shape[k];
  Buf out(t.dtype(), product(shape));
  std::vector<size_t> at(rank, 0);
  const char* from = (const char*)t.data.data();
  char* to = (char*)out.data();
  for (size_t e = 0; e < out.n; ++e) {
    size_t off = 0;
    for (size_t k = 0; k < rank; ++k) off += (op.starts[k] + at[k]) * stride[k];
    std::memcpy(to + e * es, from + off * es, es);
    for (size_t k = rank; k-- > 0;) {
      if (++at[k] < shape[k]) break;
      at[k] = 0;
    }
  }
  return Tensor(shape, std::move(out));
}

// ---- fused attention (the device's own rewrite, no counterpart in rg) ----
//
// rg's attention layer and its autodiff leave this pattern in the optimised graph (per layer):
//   S = matmul_t(q, k; tb)  S1 = S / c  Z = where(mask, S1, fill)  m = max(Z, -1, keepdims)
//   E = exp(Z - m)  s = sum(E, -1, keepdims)  P = E / s  O = P @ v
//   dv = matmul_t(P, dO; ta)  dP = matmul_t(dO, v; tb)
//   dE = dP / s + sum(((-dP) * E) / (s * s), -1, keepdims)  dS = where(mask, dE * E, 0) / c
//   dq = matmul_t(dS, transpose(k); tb)  dk = transpose(matmul_t(q, dS; ta))
// It becomes AttnFwd / AttnBwd (q, k, v, the (T, T) mask; O and dq, dk, dv as slices of their
// packed results), so the (..., T, T) tensors between them are never materialised. Values agree
// with the pattern's to rounding: softmax sums and products run in another order.
//
// Which attentions are fused: RGC_FUSED_ATTENTION=1 fuses every match and =0 none. By default
// the device fuses the shapes its tensor-core kernels take (attention.cu) where they measured
// faster than the unfused plan on a B200: sequence length 128 or 256 with head size 32 (a d256
// step of 8 heads: 9.23 against 10.32 ms) and length 256 with head size 64 (a d512 step: 273.7
// against 280.2 ms). Length 128 with head size 64 has not been measured and stays unfused.
enum class AttnFuse { None, Default, All };
AttnFuse fused_attention_mode() {
  const char* e = getenv("RGC_FUSED_ATTENTION");
  if (e && std::string(e) == "1") return AttnFuse::All;
  if (e && std::string(e) == "0") return AttnFuse::None;
  return AttnFuse::Default;
}
bool fused_attention_enabled() { return fused_attention_mode() != AttnFuse::None; }
bool fuse_by_default(size_t t, size_t d, size_t dv) { return dv == d && (((t == 128 || t == 256) && d == 32) || (t == 256 && d == 64)); }

struct AttnMatch {
  uint32_t q, k, v, O, dO, dv, dq, dk;
  uint32_t mask_src = UINT32_MAX;  // a (T, T) node (the source of a broadcast), else:
  TensorP mask_const;              // a (T, T) constant cut from a folded full-size mask
  double c = 1, fill = 0;
};

std::optional<AttnMatch> match_attention(const Graph& g, uint32_t o_id, const std::vector<std::vector<uint32_t>>& users,
                                         const std::vector<bool>& live) {
  auto node = [&](uint32_t id) -> const Node& { return g.nodes[id]; };
  auto is = [&](uint32_t id, OpKind k) { return node(id).op.kind == k; };
  auto reduce_last = [&](uint32_t id, ReduceKind r) {
    const Node& n = node(id);
    return n.op.kind == OpKind::Reduce && n.op.reduce == r && n.op.flag_a && !n.shape.empty() && n.op.shape.size() == 1 &&
           n.op.shape[0] + 1 == n.shape.size();
  };
  auto splat_of = [&](uint32_t id) -> std::optional<double> {
    if (auto v = splat(g, id)) return v;
    if (is(id, OpKind::BroadcastTo)) return splat(g, node(id).inputs[0]);
    return std::nullopt;
  };
  auto user = [&](uint32_t id, const std::function<bool(uint32_t)>& pred) -> std::optional<uint32_t> {
    std::optional<uint32_t> found;
    for (uint32_t u : users[id])
      if (live[u] && pred(u)) {
        if (found) return std::nullopt;  // ambiguous
        found = u;
      }
    return found;
  };
  const Node& on = node(o_id);
  if (!is(o_id, OpKind::MatMul) || on.dtype != DType::F32 || on.inputs.size() != 2) return std::nullopt;
  AttnMatch a;
  a.O = o_id;
  const uint32_t P = on.inputs[0];
  a.v = on.inputs[1];
  if (!is(P, OpKind::Div)) return std::nullopt;
  const uint32_t E = node(P).inputs[0], s = node(P).inputs[1];
  if (!reduce_last(s, ReduceKind::Sum) || node(s).inputs[0] != E || !is(E, OpKind::Exp)) return std::nullopt;
  const uint32_t Zm = node(E).inputs[0];
  if (!is(Zm, OpKind::Sub)) return std::nullopt;
  const uint32_t Z = node(Zm).inputs[0], m = node(Zm).inputs[1];
  if (!reduce_last(m, ReduceKind::Max) || node(m).inputs[0] != Z || !is(Z, OpKind::Where)) return std::nullopt;
  const uint32_t cond = node(Z).inputs[0], S1 = node(Z).inputs[1], fill = node(Z).inputs[2];
  if (!is(S1, OpKind::Div)) return std::nullopt;
  const uint32_t S = node(S1).inputs[0], cn = node(S1).inputs[1];
  const Node& sn = node(S);
  if (sn.op.kind != OpKind::MatMulT || sn.op.flag_a || !sn.op.flag_b) return std::nullopt;
  a.q = sn.inputs[0];
  a.k = sn.inputs[1];
  auto c = splat_of(cn);
  auto f = splat_of(fill);
  if (!c || !f) return std::nullopt;
  a.c = *c;
  a.fill = *f;
  // Shapes: q, k (..., T, d), v (..., T, dv), S (..., T, T), same leading extents.
  const auto &qs = g.shape(a.q), &ks = g.shape(a.k), &vs = g.shape(a.v), &Ss = sn.shape;
  const size_t r = qs.size();
  if (r < 2 || ks != qs || vs.size() != r || Ss.size() != r || g.dtype(a.q) != DType::F32) return std::nullopt;
  const size_t T = qs[r - 2];
  for (size_t i = 0; i + 1 < r; ++i)
    if (vs[i] != qs[i]) return std::nullopt;
  if (Ss[r - 1] != T || Ss[r - 2] != T) return std::nullopt;
  // The mask: one (T, T) pattern for every batch entry.
  const std::vector<size_t> tt{T, T};
  if (is(cond, OpKind::BroadcastTo) && g.shape(node(cond).inputs[0]) == tt) {
    a.mask_src = node(cond).inputs[0];
  } else if (is(cond, OpKind::Const) && g.shape(cond) == Ss) {
    const Tensor& full = *node(cond).op.value;
    Buf b(full.dtype(), T * T);
    for (size_t i = 0; i < T * T; ++i) b.f32()[i] = (float)full.data.get(i);
    for (size_t i = T * T; i < full.n(); ++i)
      if (!(full.data.get(i) == full.data.get(i % (T * T)))) return std::nullopt;
    a.mask_const = std::make_shared<const Tensor>(tt, std::move(b));
  } else {
    return std::nullopt;
  }
  if (g.dtype(cond) != DType::F32) return std::nullopt;
  // Backward: dv = P^T dO, dP = dO v^T, then the softmax gradient chain down to dS.
  auto dvn = user(P, [&](uint32_t u) { const Node& n = node(u); return n.op.kind == OpKind::MatMulT && n.op.flag_a && !n.op.flag_b && n.inputs[0] == P; });
  if (!dvn) return std::nullopt;
  a.dv = *dvn;
  a.dO = node(a.dv).inputs[1];
  if (g.shape(a.dO) != vs) return std::nullopt;
  auto dPn = user(a.dO, [&](uint32_t u) { const Node& n = node(u); return n.op.kind == OpKind::MatMulT && !n.op.flag_a && n.op.flag_b && n.inputs[0] == a.dO && n.inputs[1] == a.v; });
  if (!dPn) return std::nullopt;
  const uint32_t dP = *dPn;
  auto t1 = user(dP, [&](uint32_t u) { return is(u, OpKind::Div) && node(u).inputs[0] == dP && node(u).inputs[1] == s; });
  auto t2 = user(dP, [&](uint32_t u) { return is(u, OpKind::Neg); });
  if (!t1 || !t2) return std::nullopt;
  auto t3 = user(*t2, [&](uint32_t u) { const Node& n = node(u); return n.op.kind == OpKind::Mul && (n.inputs[0] == E || n.inputs[1] == E); });
  if (!t3) return std::nullopt;
  auto t4 = user(*t3, [&](uint32_t u) {
    const Node& n = node(u);
    if (n.op.kind != OpKind::Div || n.inputs[0] != *t3) return false;
    const Node& d = node(n.inputs[1]);
    return d.op.kind == OpKind::Mul && d.inputs[0] == s && d.inputs[1] == s;
  });
  if (!t4) return std::nullopt;
  auto t5 = user(*t4, [&](uint32_t u) { return reduce_last(u, ReduceKind::Sum); });
  if (!t5) return std::nullopt;
  auto dE = user(*t5, [&](uint32_t u) {
    const Node& n = node(u);
    return n.op.kind == OpKind::Add && ((n.inputs[0] == *t1 && n.inputs[1] == *t5) || (n.inputs[0] == *t5 && n.inputs[1] == *t1));
  });
  if (!dE) return std::nullopt;
  auto dZm = user(*dE, [&](uint32_t u) { const Node& n = node(u); return n.op.kind == OpKind::Mul && (n.inputs[0] == E || n.inputs[1] == E); });
  if (!dZm) return std::nullopt;
  // dS = where(mask, dZm, 0) / c, possibly computed more than once (full-size zero constants
  // are not merged by common-subexpression elimination): every copy counts.
  std::vector<uint32_t> dS;
  for (uint32_t w : users[*dZm]) {
    const Node& n = node(w);
    if (!live[w] || n.op.kind != OpKind::Where || n.inputs[1] != *dZm || n.inputs[0] != cond) continue;
    auto z = splat_of(n.inputs[2]);
    if (!z || *z != 0.0) continue;
    for (uint32_t u : users[w]) {
      const Node& dn = node(u);
      auto cc = dn.inputs.size() == 2 ? splat_of(dn.inputs[1]) : std::nullopt;
      if (live[u] && dn.op.kind == OpKind::Div && dn.inputs[0] == w && cc && *cc == a.c) dS.push_back(u);
    }
  }
  if (dS.empty()) return std::nullopt;
  auto any_user = [&](const std::function<bool(uint32_t, uint32_t)>& pred) -> std::optional<uint32_t> {
    std::optional<uint32_t> found;
    for (uint32_t d : dS)
      for (uint32_t u : users[d])
        if (live[u] && pred(u, d)) {
          if (found && *found != u) return std::nullopt;  // ambiguous
          found = u;
        }
    return found;
  };
  auto swaps_last2 = [&](uint32_t id) {
    const Node& n = node(id);
    if (n.op.kind != OpKind::Transpose || n.op.shape.size() != r) return false;
    for (size_t i = 0; i < r; ++i)
      if (n.op.shape[i] != (i + 2 < r ? i : (i + 2 == r ? r - 1 : r - 2))) return false;
    return true;
  };
  auto dqn = any_user([&](uint32_t u, uint32_t d) {
    const Node& n = node(u);
    if (n.inputs.size() != 2 || n.inputs[0] != d) return false;
    if (n.op.kind == OpKind::MatMul) return n.inputs[1] == a.k;
    return n.op.kind == OpKind::MatMulT && !n.op.flag_a && n.op.flag_b && swaps_last2(n.inputs[1]) && node(n.inputs[1]).inputs[0] == a.k;
  });
  if (!dqn) return std::nullopt;
  a.dq = *dqn;
  auto dkT = any_user([&](uint32_t u, uint32_t d) {
    const Node& n = node(u);
    return n.op.kind == OpKind::MatMulT && n.op.flag_a && !n.op.flag_b && n.inputs.size() == 2 && n.inputs[0] == a.q && n.inputs[1] == d;
  });
  if (!dkT) return std::nullopt;
  auto dkn = user(*dkT, [&](uint32_t u) { return swaps_last2(u); });
  if (!dkn) return std::nullopt;
  a.dk = *dkn;
  return a;
}

struct Simplified;
Simplified fuse_attention(const Simplified& s);

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
    if (concat_pads && op.kind == OpKind::Slice && ins.size() == 1) {
      if (auto folded = slice_of_constant(ng, ins[0], op, node.shape)) {
        op = Op::make(OpKind::Const);
        op.value = std::make_shared<const Tensor>(std::move(*folded));
        ins.clear();
        r.st.folded += 1;
      }
    }
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

// The packed form of a matched attention (graph.h): q, k and v are the three parts of one
// (B, T, 3, H, d) tensor, split by transpose (2, 0, 3, 1, 4) and a slice each (through reshapes);
// dO is a (B, T, H, d) tensor under transpose (0, 2, 1, 3); and dq, dk, dv are used only to be
// joined back: reshaped, concatenated on axis 0 and transposed by (1, 3, 0, 2, 4). The fused ops
// then read and write the packed tensors, and the head-split and head-join copies go away. Only
// for the shapes of the tensor-core kernels (length 128 or 256, head size 32 or 64).
struct AttnPacked {
  uint32_t qkv = 0, dO = 0, grad = 0;  // grad: the transpose whose value is the gradient of qkv
  size_t heads = 0;
};

std::optional<AttnPacked> packed_attention(const Graph& g, const AttnMatch& m, const std::vector<std::vector<uint32_t>>& users,
                                           const std::vector<bool>& live) {
  auto strip = [&](uint32_t id) {
    while (g.nodes[id].op.kind == OpKind::Reshape) id = g.nodes[id].inputs[0];
    return id;
  };
  auto transpose_of = [&](uint32_t id, const std::vector<size_t>& perm) {
    const Node& n = g.nodes[id];
    return n.op.kind == OpKind::Transpose && n.op.shape == perm && n.inputs.size() == 1;
  };
  // The single live user of `id`, or none.
  auto only_user = [&](uint32_t id) -> std::optional<uint32_t> {
    std::optional<uint32_t> found;
    for (uint32_t u : users[id])
      if (live[u]) {
        if (found) return std::nullopt;
        found = u;
      }
    return found;
  };
  const auto& qs = g.shape(m.q);
  if (qs.size() != 4 || g.shape(m.k) != qs || g.shape(m.v) != qs) return std::nullopt;
  const size_t B = qs[0], H = qs[1], T = qs[2], d = qs[3];
  if (!((T == 128 || T == 256) && (d == 32 || d == 64))) return std::nullopt;
  AttnPacked p;
  p.heads = H;
  uint32_t split = UINT32_MAX;
  const uint32_t parts[3] = {m.q, m.k, m.v};
  for (size_t w = 0; w < 3; ++w) {
    const uint32_t sl = strip(parts[w]);
    const Node& n = g.nodes[sl];
    if (n.op.kind != OpKind::Slice || n.inputs.size() != 1 || !transpose_of(n.inputs[0], {2, 0, 3, 1, 4})) return std::nullopt;
    const std::vector<size_t> ts = {3, B, H, T, d};
    if (g.shape(n.inputs[0]) != ts) return std::nullopt;
    std::vector<size_t> starts(5, 0), stops = ts;
    starts[0] = w;
    stops[0] = w + 1;
    if (n.op.starts != starts || n.op.stops != stops) return std::nullopt;
    if (split != UINT32_MAX && split != n.inputs[0]) return std::nullopt;
    split = n.inputs[0];
  }
  p.qkv = g.nodes[split].inputs[0];
  const std::vector<size_t> packed = {B, T, 3, H, d};
  if (g.shape(p.qkv) != packed || g.nodes[p.qkv].dtype != DType::F32) return std::nullopt;
  const uint32_t dt = strip(m.dO);
  if (!transpose_of(dt, {0, 2, 1, 3})) return std::nullopt;
  p.dO = g.nodes[dt].inputs[0];
  if (g.shape(p.dO) != std::vector<size_t>{B, T, H, d}) return std::nullopt;
  // dq, dk, dv: each used once, through reshapes, by one concat on axis 0 in that order.
  std::optional<uint32_t> cat;
  const uint32_t grads[3] = {m.dq, m.dk, m.dv};
  for (size_t w = 0; w < 3; ++w) {
    uint32_t id = grads[w];
    std::optional<uint32_t> u = only_user(id);
    while (u && g.nodes[*u].op.kind == OpKind::Reshape) {
      id = *u;
      u = only_user(id);
    }
    if (!u || g.nodes[*u].op.kind != OpKind::Concat || g.nodes[*u].op.index != 0) return std::nullopt;
    const Node& c = g.nodes[*u];
    if (c.inputs.size() != 3 || c.inputs[w] != id || strip(c.inputs[w]) != grads[w]) return std::nullopt;
    if (cat && *cat != *u) return std::nullopt;
    cat = *u;
  }
  auto t = only_user(*cat);
  if (!t || !transpose_of(*t, {1, 3, 0, 2, 4}) || g.shape(*t) != packed) return std::nullopt;
  p.grad = *t;
  return p;
}

// `gpu`: planning for the device, which recomputes forward values inside the backward groups
// that read them (recompute_in_consumers) and keeps every other activation while the peak live
// bytes stay within DEVICE_ACTIVATIONS_BYTES; above it rg's policy, escalating to transcendental
// values when that plan still peaks above the same bound.

// Rebuilds the graph with every matched attention replaced (see match_attention).
Simplified fuse_attention(const Simplified& in) {
  const Graph& g = in.g;
  const size_t N = g.nodes.size();
  auto live = g.reachable(in.out);
  std::vector<std::vector<uint32_t>> users(N);
  for (size_t i = 0; i < N; ++i)
    if (live[i])
      for (auto x : g.nodes[i].inputs) users[x].push_back((uint32_t)i);
  std::vector<AttnMatch> matches;
  std::vector<std::optional<AttnPacked>> packs;
  std::vector<long> match_of(N, -1);  // O, dv, dq, dk node -> match index
  for (size_t i = 0; i < N; ++i) {
    if (!live[i] || match_of[i] >= 0) continue;
    auto m = match_attention(g, (uint32_t)i, users, live);
    if (!m || match_of[m->dv] >= 0 || match_of[m->dq] >= 0 || match_of[m->dk] >= 0) continue;
    if (fused_attention_mode() == AttnFuse::Default) {
      const auto& qs = g.shape(m->q);
      if (!fuse_by_default(qs[qs.size() - 2], qs.back(), g.shape(m->v).back())) continue;
    }
    for (uint32_t id : {m->O, m->dv, m->dq, m->dk}) match_of[id] = (long)matches.size();
    matches.push_back(*m);
    packs.push_back(packed_attention(g, *m, users, live));
  }
  if (matches.empty()) return in;
  Simplified r;
  r.st = in.st;
  Graph& ng = r.g;
  std::vector<uint32_t> map(N, UINT32_MAX);
  std::vector<uint32_t> stats(matches.size(), UINT32_MAX), mask(matches.size(), UINT32_MAX);
  std::vector<bool> grads_done(matches.size(), false);
  std::vector<bool>& backward = r.backward;
  auto slice_last = [&](uint32_t src, size_t from, size_t to) {
    const auto& sh = ng.shape(src);
    Op sl = Op::make(OpKind::Slice);
    sl.starts.assign(sh.size(), 0);
    sl.stops = sh;
    sl.starts.back() = from;
    sl.stops.back() = to;
    return ng.add(sl, {src});
  };
  auto values = [&](const AttnMatch& m, size_t heads) {
    const size_t n = heads ? 3 : 2;
    Buf b(DType::F64, n);
    b.f64()[0] = m.c;
    b.f64()[1] = m.fill;
    if (heads) b.f64()[2] = (double)heads;
    return std::make_shared<const Tensor>(std::vector<size_t>{n}, std::move(b));
  };
  auto mark = [&](bool bw) { backward.resize(ng.nodes.size(), bw); };
  for (size_t i = 0; i < N; ++i) {
    const Node& node = g.nodes[i];
    ng.cur_source = node.source;
    ng.cur_origin.reset();
    if (node.op.kind == OpKind::Input) {
      map[i] = ng.input(node.shape, node.dtype);
      ng.nodes[map[i]].op = node.op;
      mark(false);
      continue;
    }
    const long mi = match_of[i];
    if (mi >= 0 && matches[mi].O == i) {
      const AttnMatch& m = matches[mi];
      if (m.mask_src != UINT32_MAX) mask[mi] = map[m.mask_src];
      else mask[mi] = ng.constant(m.mask_const);
      mark(false);
      Op f = Op::make(OpKind::AttnFwd);
      const auto& pk = packs[mi];
      f.value = values(m, pk ? pk->heads : 0);
      uint32_t a = pk ? ng.add(f, {map[pk->qkv], mask[mi]}) : ng.add(f, {map[m.q], map[m.k], map[m.v], mask[mi]});
      const size_t dv = g.shape(m.v).back();
      map[i] = slice_last(a, 0, dv);
      stats[mi] = a;  // the backward reads O and the row statistics from the packed output
      mark(false);
      r.st.simplified += 1;
      continue;
    }
    if (mi >= 0) {
      const AttnMatch& m = matches[mi];
      if (!grads_done[mi] && packs[mi]) {
        // Packed: the gradient of qkv directly; dq, dk, dv and their join are not rebuilt.
        const auto& pk = *packs[mi];
        Op b = Op::make(OpKind::AttnBwd);
        b.value = values(m, pk.heads);
        map[pk.grad] = ng.add(b, {map[pk.qkv], mask[mi], stats[mi], map[pk.dO]});
        mark(true);
        grads_done[mi] = true;
      }
      if (!grads_done[mi]) {
        Op b = Op::make(OpKind::AttnBwd);
        b.value = values(m, 0);
        uint32_t gid = ng.add(b, {map[m.q], map[m.k], map[m.v], mask[mi], stats[mi], map[m.dO]});
        const size_t d = g.shape(m.q).back(), dv = g.shape(m.v).back();
        uint32_t dq = slice_last(gid, 0, d), dk = slice_last(gid, d, 2 * d), dvv = slice_last(gid, 2 * d, 2 * d + dv);
        mark(true);
        map[m.dq] = dq;
        map[m.dk] = dk;
        map[m.dv] = dvv;
        grads_done[mi] = true;
      }
      continue;
    }
    if (map[i] != UINT32_MAX) continue;  // the gradient of a packed attention's qkv, already built
    std::vector<uint32_t> ins;
    bool ok = true;
    for (auto x : node.inputs) {
      ok = ok && map[x] != UINT32_MAX;
      ins.push_back(map[x]);
    }
    if (!ok) continue;  // depends on a node that was replaced before its inputs existed (never live)
    uint32_t id = node.op.kind == OpKind::Const ? ng.constant(node.op.value) : ng.add(node.op, ins);
    ng.nodes[id].origin = node.origin;
    mark(i < in.backward.size() && in.backward[i]);
    backward[id] = i < in.backward.size() && in.backward[i];
    map[i] = id;
  }
  for (auto o : in.out) r.out.push_back(map[o]);
  backward.resize(ng.nodes.size(), false);
  return r;
}

OptResult finish(const Graph& ng, const std::vector<uint32_t>& out, const std::vector<bool>& backward, OptStats st, bool gpu = false) {
  if (gpu) {
    OptStats rs = st;
    auto rc = recompute_in_consumers(ng, out, backward, rs);
    if (Plan::build(rc.first, rc.second, true).peak_live_bytes <= DEVICE_ACTIVATIONS_BYTES) {
      rs.nodes_after = count_kept(rc.first, rc.second);
      return OptResult{std::move(rc.first), std::move(rc.second), rs};
    }
  }
  auto hr = rematerialize(ng, out, backward, REMAT_MIN, false, st);
  if (Plan::build(hr.first, hr.second, true).peak_live_bytes > (gpu ? DEVICE_ACTIVATIONS_BYTES : COSTLY_REMAT_ABOVE_BYTES)) {
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
    if (gpu && fused_attention_enabled()) s = fuse_attention(s);
    return finish(s.g, s.out, s.backward, s.st, gpu);
  }
  Simplified baseline = simplify(g, outputs, true, gpu);
  Simplified first = simplify(g, outputs, false);
  size_t before = count_kept(g, outputs);
  if (mode == OptMode::SearchLinear && !has_matrix_structure(first.g, first.out)) {
    baseline.st.nodes_before = before;
    if (gpu && fused_attention_enabled()) baseline = fuse_attention(baseline);
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
  if (gpu && fused_attention_enabled()) chosen = fuse_attention(chosen);
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
