// Graph rewrites before planning (restates src/optimize.rs): constant folding, identities,
// pow(x,2) -> x*x, dropping materialised broadcasts into binary ops, transposes folded into
// matmul flags, common-subexpression elimination and rematerialisation.
#pragma once
#include <optional>
#include <string>

#include "graph.h"

namespace rg {

enum class OptMode { None, Standard, SearchExact, SearchLinear, Search, Auto };
bool parse_opt_mode(const std::string& s, OptMode* m);

struct SearchStats {
  bool accepted = false;
  size_t iterations = 0, egraph_nodes = 0;
  double cost_before = 0, cost_after = 0;
};

struct OptStats {
  size_t nodes_before = 0, nodes_after = 0, folded = 0, simplified = 0, cse = 0, rematerialized = 0;
  std::optional<SearchStats> search;
  Json json() const;
};

struct OptResult {
  Graph graph;
  std::vector<uint32_t> outputs;
  OptStats stats;
};

OptResult optimize(const Graph& g, const std::vector<uint32_t>& outputs);
// `gpu` selects the GPU cost model for the search modes (rg: the Metal model on its GPU).
OptResult optimize_mode(const Graph& g, const std::vector<uint32_t>& outputs, OptMode mode, bool gpu = false);
bool has_matrix_structure(const Graph& g, const std::vector<uint32_t>& outputs);

// Estimated nanoseconds per node (egraph.rs:170-233); only ratios matter.
struct CostModel {
  double per_op, per_element, per_flop, per_math_element, per_transpose_element;
  static const CostModel CPU, METAL, CUDA;
  double node(const Op& op, const std::vector<size_t>& shape, const std::vector<const std::vector<size_t>*>& args) const;
  // Whole-graph cost, shared values counted once; nodes whose inputs are all constants are free.
  double graph_cost(const Graph& g, const std::vector<uint32_t>& outputs) const;
};

// Equality saturation (egraph.rs:367-427): a cheaper graph computing the same outputs under the
// rule set (0 exact, 1 linear: + matrix-product reassociation and factoring, 2 rounding: +
// elementwise associativity and distribution), if the search finds one.
std::optional<std::pair<Graph, std::vector<uint32_t>>> search(const Graph& g, const std::vector<uint32_t>& outputs, const CostModel& model,
                                                              int rule_set, size_t iter_limit, size_t node_limit, SearchStats* st);

}  // namespace rg
