// mcke/graph/cost_model.hpp -- a roofline lower bound for an op and a graph.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/cost_model.hpp (the
// roofline time of one OpCost, and the whole-graph ratio its banner defines):
// each node is judged against the roof that binds it,
//     node_ms = max(flops / peak_flops, bytes / peak_bandwidth),
// and a graph's sequential lower bound is the sum over its nodes.  Divided by
// the measured time of a run this gives the reference's cost-model ratio: near
// 1.0 the graph runs as fast as its parts allow; above 1.0 streams or devices
// overlapped nodes.  Host arithmetic only.
#pragma once

#include <algorithm>

#include "mcke/graph/graph.hpp"
#include "mcke/graph/op.hpp"

namespace mcke {

struct Roofline {
  double peak_flops_per_s = 0.0;  // e.g. the measured bf16 tensor rate
  double peak_bytes_per_s = 0.0;  // e.g. the measured HBM copy rate
};

// Lower bound on one op's time in milliseconds; 0 for a zero-cost op or a
// roofline with a zero field.
[[nodiscard]] inline double roofline_ms(const OpCost& c, const Roofline& r) {
  const double tf = r.peak_flops_per_s > 0.0 ? static_cast<double>(c.flops) / r.peak_flops_per_s : 0.0;
  const double tb = r.peak_bytes_per_s > 0.0 ? static_cast<double>(c.bytes) / r.peak_bytes_per_s : 0.0;
  return std::max(tf, tb) * 1e3;
}

// Sum over the graph's nodes of roofline_ms(node cost on the graph's global
// shapes): the sequential lower bound of one run on one device.  A graph
// sharded over D devices has about 1/D of it per device.
[[nodiscard]] inline double graph_roofline_ms(const Graph& g, const Roofline& r) {
  double ms = 0.0;
  for (std::size_t n = 0; n < g.num_nodes(); ++n) {
    const Node& node = g.node(static_cast<NodeId>(n));
    std::vector<TensorDesc> in;
    in.reserve(node.inputs.size());
    for (TensorId t : node.inputs) in.push_back(g.tensor(t));
    ms += roofline_ms(node.op->cost(in), r);
  }
  return ms;
}

}  // namespace mcke
