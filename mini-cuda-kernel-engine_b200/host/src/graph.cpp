// graph.cpp -- Graph construction and topological order.
#include "mcke/graph/graph.hpp"

#include <algorithm>
#include <deque>

namespace mcke {

TensorId Graph::add_input(TensorDesc desc) {
  const auto id = static_cast<TensorId>(tensors_.size());
  tensors_.push_back(std::move(desc));
  producer_.push_back(kInvalidNode);
  consumers_.emplace_back();
  finalized_ = false;
  return id;
}

StatusOr<std::vector<TensorId>> Graph::add_node(std::string name, OpPtr op, std::vector<TensorId> inputs) {
  if (!op) return InvalidArgumentError("add_node(" + name + "): null op");
  std::vector<TensorDesc> in;
  for (TensorId t : inputs) {
    if (t >= tensors_.size()) return InvalidArgumentError("add_node(" + name + "): unknown input tensor");
    in.push_back(tensors_[t]);
  }
  auto outs = op->infer(in);
  if (!outs.ok()) return Status(outs.status().code(), "node '" + name + "': " + outs.status().message());
  const auto nid = static_cast<NodeId>(nodes_.size());
  Node node;
  node.id = nid;
  node.name = std::move(name);
  node.op = std::move(op);
  node.inputs = inputs;
  for (TensorId t : inputs) consumers_[t].push_back(nid);
  for (auto& d : *outs) {
    if (d.name.empty()) d.name = node.name + ".out" + std::to_string(node.outputs.size());
    const auto id = static_cast<TensorId>(tensors_.size());
    tensors_.push_back(d);
    producer_.push_back(nid);
    consumers_.emplace_back();
    node.outputs.push_back(id);
  }
  std::vector<TensorId> result = node.outputs;
  nodes_.push_back(std::move(node));
  finalized_ = false;
  return result;
}

Status Graph::mark_output(TensorId t) {
  if (t >= tensors_.size()) return InvalidArgumentError("mark_output: unknown tensor");
  if (!is_output(t)) outputs_.push_back(t);
  return OkStatus();
}

bool Graph::is_output(TensorId t) const {
  return std::find(outputs_.begin(), outputs_.end(), t) != outputs_.end();
}

// FIFO Kahn: among ready nodes, insertion order -- deterministic and, for the
// fan-out graphs the executor overlaps, breadth-first across branches.
Status Graph::finalize() {
  if (outputs_.empty()) return FailedPreconditionError("finalize: no tensor is marked as an output");
  std::vector<int> pending(nodes_.size(), 0);
  for (const Node& n : nodes_)
    for (TensorId t : n.inputs)
      if (producer_[t] != kInvalidNode) ++pending[n.id];
  std::deque<NodeId> ready;
  for (const Node& n : nodes_)
    if (pending[n.id] == 0) ready.push_back(n.id);
  order_.clear();
  while (!ready.empty()) {
    const NodeId id = ready.front();
    ready.pop_front();
    order_.push_back(id);
    for (TensorId t : nodes_[id].outputs)
      for (NodeId c : consumers_[t])
        if (--pending[c] == 0) ready.push_back(c);
  }
  if (order_.size() != nodes_.size()) return InternalError("finalize: the graph has a cycle");
  finalized_ = true;
  return OkStatus();
}

std::string Graph::to_dot() const {
  std::string s = "digraph mcke {\n";
  for (const Node& n : nodes_) {
    s += "  n" + std::to_string(n.id) + " [label=\"" + n.name + "\\n" + std::string(n.op->type_name()) + "\"];\n";
    for (TensorId t : n.inputs)
      if (producer_[t] != kInvalidNode)
        s += "  n" + std::to_string(producer_[t]) + " -> n" + std::to_string(n.id) + ";\n";
  }
  return s + "}\n";
}

}  // namespace mcke
