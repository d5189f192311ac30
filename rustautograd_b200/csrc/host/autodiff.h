// Reverse-mode differentiation emitting ordinary IR nodes (restates src/autodiff.rs).
#pragma once
#include "graph.h"

namespace rg {

// Appends d(y)/d(wrts) to the graph and records them in `g.grads` (autodiff.rs:246-326).
std::vector<uint32_t> grad(Graph& g, uint32_t y, const std::vector<uint32_t>& wrts);

}  // namespace rg
