// SSA intermediate representation with shape and dtype inference (restates src/graph.rs).
//
// Every value is a node; inputs are node ids of earlier nodes, so a graph is already in
// topological order. Errors are structured JSON diagnostics thrown as `DiagError`.
#pragma once
#include <cstdint>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <utility>
#include <vector>

#include "json.h"
#include "tensor.h"

namespace rg {

struct Plan;
struct Fuse;
struct Body;
using BodyP = std::shared_ptr<Body>;

enum class ReduceKind : uint8_t { Sum = 0, Max = 1, Min = 2 };

// graph.rs:47-114. The numbering is part of the plan wire format (include/rgc.h).
enum class OpKind : uint8_t {
  Input = 0, Const, Neg, Exp, Log, Sqrt, Sin, Cos, Tanh, Abs, Sign,
  Add, Sub, Mul, Div, Pow, Max, Min, Gt, Ge, Where,
  MatMul, MatMulT, Reduce, Reshape, Transpose, BroadcastTo, Slice, Pad, Cast,
  StopGradient, Floor, Take, TakeAlong, TakeGrad, TakeAlongGrad, Concat, Argmax,
  RandUniform, RandNormal, KeySplit, ArgTopK, Cumsum, Scan, While, Cond, Output,
  Placeholder, Custom,
  // Data parallelism (no counterpart in rg): the sum of a value over all ranks.
  AllReduce,
  // Fused attention (no counterpart in rg; produced only by the device's graph rewrite).
  // AttnFwd(q, k, v, mask) with value = [c, fill]: per batch entry, Z = where(mask, q k^T / c,
  // fill), softmax along the last axis (max-subtracted), O = P v; the result packs O with each
  // row's max and exp-sum: (..., T, dv + 2). AttnBwd(q, k, v, mask, fwd, dO), with `fwd` that
  // packed forward output: the gradients of O with respect to q, k and v for the cotangent dO,
  // packed as (..., T, 2 d + dv). With P the softmax rebuilt from the row statistics and
  // D = rowsum(dO * O): dS = P (dO v^T - D) / c where the mask is nonzero (0 elsewhere),
  // dq = dS k, dk = dS^T q, dv = P^T dO.
  // Packed form, value = [c, fill, H]: AttnFwd(qkv, mask) and AttnBwd(qkv, mask, fwd, dO) with
  // qkv the (B, T, 3, H, d) projection output before the head split (batch entry b * H + h) and
  // dO (B, T, H, d) before the head merge is undone; AttnFwd still gives (B, H, T, d + 2) and
  // AttnBwd gives the gradient of qkv, (B, T, 3, H, d). No head-split copies are needed.
  AttnFwd,
  AttnBwd,
};

struct Op {
  OpKind kind = OpKind::Input;
  // Attributes; which ones are meaningful depends on `kind`.
  size_t index = 0;             // Input(k), Output{index}, Take/Concat/TakeGrad axis, ArgTopK k, KeySplit n
  std::vector<size_t> shape;    // Reshape/BroadcastTo/Pad/TakeGrad/TakeAlongGrad/Rand*/Output shape; Transpose perm; Reduce axes
  std::vector<size_t> starts;   // Slice/Pad
  std::vector<size_t> stops;    // Slice
  DType dtype = DType::F32;     // Cast, Rand*, Output
  bool flag_a = false;          // MatMulT ta, Reduce keepdims, Cumsum/Scan reverse
  bool flag_b = false;          // MatMulT tb
  ReduceKind reduce = ReduceKind::Sum;
  TensorP value;                // Const
  BodyP body, body2;            // Scan body / While cond+body / Cond then+else
  size_t n_carry = 0, n_x = 0, length = 0, max_iterations = 0;
  uint32_t placeholder = 0;     // Custom
  std::vector<std::pair<uint32_t, uint32_t>> rules;  // Custom

  static Op make(OpKind k) {
    Op o;
    o.kind = k;
    return o;
  }
  const char* name() const;
  bool is_unary_elementwise() const;
  bool is_binary_elementwise() const;
  bool is_control_flow() const { return kind == OpKind::Scan || kind == OpKind::While || kind == OpKind::Cond; }
  bool int_ok() const;
  bool is_nonsmooth() const;
  // Key for common-subexpression elimination: equal keys mean interchangeable nodes
  // (optimize.rs:395, which keys on the op's debug form and its inputs).
  std::string key() const;
};

struct Node {
  Op op;
  std::vector<uint32_t> inputs;
  std::vector<size_t> shape;
  DType dtype = DType::F32;
  std::shared_ptr<const std::string> source;
  std::optional<uint32_t> origin;  // forward node whose VJP produced this node
  size_t n() const { return product(shape); }
};

struct GradRecord {
  uint32_t y, wrt, grad;
};

struct DiagError : std::exception {
  Json diag;
  std::string text;
  explicit DiagError(Json d) : diag(std::move(d)), text(diag.dump()) {}
  const char* what() const noexcept override { return text.c_str(); }
};

// graph.rs:203-212
Json diag(const std::string& code, const std::string& severity, Json node, Json observation,
          const std::string& cause, const std::string& certainty);

// graph.rs:214-226; returns false when the shapes do not broadcast.
bool broadcast_shapes(const std::vector<size_t>& a, const std::vector<size_t>& b, std::vector<size_t>* out);

struct Graph {
  std::vector<Node> nodes;
  size_t n_inputs = 0;
  std::vector<GradRecord> grads;
  std::vector<Json> notes;
  std::shared_ptr<const std::string> cur_source;
  std::optional<uint32_t> cur_origin;

  Json node_json(uint32_t id) const;
  uint32_t input(const std::vector<size_t>& shape, DType d);
  uint32_t placeholder(const std::vector<size_t>& shape, DType d);
  uint32_t constant(Tensor t);
  uint32_t constant(TensorP t);
  uint32_t scalar(DType d, double x) { return constant(Tensor::full(d, {}, x)); }
  const std::vector<size_t>& shape(uint32_t id) const { return nodes[id].shape; }
  DType dtype(uint32_t id) const { return nodes[id].dtype; }
  // Appends a node after checking arity, dtypes and shapes (graph.rs:316-383).
  uint32_t add(Op op, const std::vector<uint32_t>& inputs);
  std::vector<bool> reachable(const std::vector<uint32_t>& outputs) const;
  Graph to_f64() const;

 private:
  uint32_t push(Op op, std::vector<uint32_t> inputs, std::vector<size_t> shape, DType d);
  Json pending_json(const Op& op) const;
  [[noreturn]] void static_err(const std::string& code, const Op& op, Json obs, const std::string& cause) const;
  std::vector<size_t> infer(const Op& op, const std::vector<std::vector<size_t>>& s) const;
  void check_control_flow(const Op& op, const std::vector<uint32_t>& inputs) const;
};

// A traced sub-function, the unit of control flow (graph.rs:11-38). `reference` keeps every
// value (diagnostics); `opt` is the optimised graph from which per-device fast plans are built.
struct Body {
  Graph graph;
  std::vector<uint32_t> outputs;
  Graph opt;
  std::vector<uint32_t> opt_outputs;
  std::shared_ptr<Plan> fast;       // Fuse::DEFAULT, as rg builds it
  std::shared_ptr<Plan> reference;  // no reuse, no fusion

  static BodyP make(Graph g, std::vector<uint32_t> outputs);
  DType output_dtype(size_t k) const { return graph.dtype(outputs[k]); }
  const std::vector<size_t>& output_shape(size_t k) const { return graph.shape(outputs[k]); }
  // The body's plan for a given fusion configuration, built once per configuration.
  std::shared_ptr<Plan> plan_for(const Fuse& f);

 private:
  std::mutex mu_;
  std::vector<std::pair<std::string, std::shared_ptr<Plan>>> cache_;
};

}  // namespace rg
