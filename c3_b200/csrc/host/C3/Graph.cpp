#include "C3/Graph.h"

#include <algorithm>
#include <sstream>
#include <stdexcept>

namespace ct {
namespace c3 {

const char* nodeName(const NodeVariant& v) {
  return std::visit([](auto&& n) -> const char* { return std::decay_t<decltype(n)>::name; }, v);
}

size_t Graph::addInput(const TensorDesc& desc) {
  Node n;
  n.id = nodes_.size();
  n.op = ConstNode{0.0};  // placeholder; membership in inputs_ marks it as an input
  n.out_desc = desc;
  nodes_.push_back(n);
  inputs_.push_back(n.id);
  return n.id;
}

size_t Graph::addNode(NodeVariant op, const std::vector<size_t>& input_ids, const TensorDesc& out_desc) {
  Node n;
  n.id = nodes_.size();
  n.op = std::move(op);
  n.inputs = input_ids;
  n.out_desc = out_desc;
  for (size_t in : input_ids) {
    if (in >= nodes_.size()) throw std::invalid_argument("Graph::addNode: unknown input id");
    nodes_[in].outputs.push_back(n.id);
  }
  nodes_.push_back(std::move(n));
  return nodes_.back().id;
}

size_t Graph::addConstant(double value, const TensorDesc& desc) {
  Node n;
  n.id = nodes_.size();
  n.op = ConstNode{value};
  n.out_desc = desc;
  nodes_.push_back(n);
  return n.id;
}

void Graph::markOutput(size_t node_id) {
  if (node_id >= nodes_.size()) throw std::invalid_argument("Graph::markOutput: unknown id");
  if (std::find(outputs_.begin(), outputs_.end(), node_id) == outputs_.end())
    outputs_.push_back(node_id);
}

bool Graph::isInput(size_t id) const {
  return std::find(inputs_.begin(), inputs_.end(), id) != inputs_.end();
}

bool Graph::isConst(size_t id) const {
  return id < nodes_.size() && !isInput(id) && std::holds_alternative<ConstNode>(nodes_[id].op);
}

bool Graph::isValid() const {
  for (const auto& n : nodes_)
    for (size_t in : n.inputs)
      if (in >= n.id) return false;
  for (size_t o : outputs_)
    if (o >= nodes_.size()) return false;
  return true;
}

std::vector<size_t> Graph::computeNodes() const {
  std::vector<size_t> ids;
  for (const auto& n : nodes_)
    if (!isInput(n.id) && !std::holds_alternative<ConstNode>(n.op)) ids.push_back(n.id);
  return ids;
}

Graph Graph::eliminateDeadCode() const {
  std::vector<bool> live(nodes_.size(), false);
  std::vector<size_t> stack(outputs_.begin(), outputs_.end());
  while (!stack.empty()) {
    const size_t id = stack.back();
    stack.pop_back();
    if (live[id]) continue;
    live[id] = true;
    for (size_t in : nodes_[id].inputs) stack.push_back(in);
  }
  for (size_t in : inputs_) live[in] = true;  // inputs keep their positions
  Graph g;
  std::vector<size_t> remap(nodes_.size(), SIZE_MAX);
  for (const auto& n : nodes_) {
    if (!live[n.id]) continue;
    if (isInput(n.id)) {
      remap[n.id] = g.addInput(n.out_desc);
    } else if (std::holds_alternative<ConstNode>(n.op)) {
      remap[n.id] = g.addConstant(std::get<ConstNode>(n.op).value, n.out_desc);
    } else {
      std::vector<size_t> ins;
      for (size_t in : n.inputs) ins.push_back(remap[in]);
      remap[n.id] = g.addNode(n.op, ins, n.out_desc);
    }
  }
  for (size_t o : outputs_) g.markOutput(remap[o]);
  return g;
}

std::string Graph::toString() const {
  std::ostringstream ss;
  ss << "Graph (" << nodes_.size() << " nodes, " << inputs_.size() << " inputs, " << outputs_.size()
     << " outputs)\n";
  for (const auto& n : nodes_) {
    ss << "  [" << n.id << "] ";
    if (isInput(n.id)) ss << "INPUT ";
    if (!isInput(n.id) && std::holds_alternative<ConstNode>(n.op))
      ss << "Const(" << std::get<ConstNode>(n.op).value << ")";
    else
      ss << nodeName(n.op);
    if (auto* s = std::get_if<SumReduceNode>(&n.op)) ss << "{axis=" << s->axis << "}";
    if (auto* t = std::get_if<TransposeNode>(&n.op)) ss << "{" << t->dim0 << "," << t->dim1 << "}";
    ss << " in(";
    for (size_t i = 0; i < n.inputs.size(); ++i) ss << (i ? "," : "") << n.inputs[i];
    ss << ") shape[";
    for (size_t i = 0; i < n.out_desc.shape.size(); ++i) ss << (i ? "x" : "") << n.out_desc.shape[i];
    ss << "]";
    if (std::find(outputs_.begin(), outputs_.end(), n.id) != outputs_.end()) ss << " OUTPUT";
    ss << "\n";
  }
  return ss.str();
}

}  // namespace c3
}  // namespace ct
