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
OptResult optimize_mode(const Graph& g, const std::vector<uint32_t>& outputs, OptMode mode);
bool has_matrix_structure(const Graph& g, const std::vector<uint32_t>& outputs);

// Matrix-product reassociation for `search-linear` (the Linear rule set of egraph.rs:148-157,
// restricted to chains of plain products): returns a cheaper equivalent graph, if any.
std::optional<std::pair<Graph, std::vector<uint32_t>>> reassociate_products(const Graph& g, const std::vector<uint32_t>& outputs, SearchStats* st);

}  // namespace rg
