// mcke/graph/graph.hpp -- the operator DAG.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/graph.hpp (TensorDesc :62,
// Node :84, Graph :109: add_input / add_node / mark_output / finalize with a
// FIFO Kahn topological order).  Shapes and dtypes are inferred when a node is
// added, so a bad graph fails at build time, naming the node.
#pragma once

#include <string>
#include <vector>

#include "mcke/graph/op.hpp"

namespace mcke {

struct Node {
  NodeId id = kInvalidNode;
  std::string name;
  OpPtr op;
  std::vector<TensorId> inputs;
  std::vector<TensorId> outputs;
};

class Graph {
 public:
  TensorId add_input(TensorDesc desc);
  [[nodiscard]] StatusOr<std::vector<TensorId>> add_node(std::string name, OpPtr op,
                                                         std::vector<TensorId> inputs);
  [[nodiscard]] Status mark_output(TensorId t);
  [[nodiscard]] Status finalize();

  [[nodiscard]] bool finalized() const noexcept { return finalized_; }
  [[nodiscard]] std::size_t num_tensors() const noexcept { return tensors_.size(); }
  [[nodiscard]] std::size_t num_nodes() const noexcept { return nodes_.size(); }
  [[nodiscard]] const TensorDesc& tensor(TensorId t) const { return tensors_.at(t); }
  [[nodiscard]] Node& node(NodeId n) { return nodes_.at(n); }
  [[nodiscard]] const Node& node(NodeId n) const { return nodes_.at(n); }
  [[nodiscard]] NodeId producer(TensorId t) const { return producer_.at(t); }
  [[nodiscard]] const std::vector<NodeId>& consumers(TensorId t) const { return consumers_.at(t); }
  [[nodiscard]] bool is_input(TensorId t) const { return producer_.at(t) == kInvalidNode; }
  [[nodiscard]] bool is_output(TensorId t) const;
  [[nodiscard]] const std::vector<TensorId>& outputs() const noexcept { return outputs_; }
  [[nodiscard]] const std::vector<NodeId>& topo_order() const noexcept { return order_; }
  [[nodiscard]] std::string to_dot() const;

 private:
  std::vector<TensorDesc> tensors_;
  std::vector<NodeId> producer_;
  std::vector<std::vector<NodeId>> consumers_;
  std::vector<Node> nodes_;
  std::vector<TensorId> outputs_;
  std::vector<NodeId> order_;
  bool finalized_ = false;
};

}  // namespace mcke
