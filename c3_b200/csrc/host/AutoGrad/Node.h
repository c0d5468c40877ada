// Autograd node shim. C3BackwardCapture keys its kernels by typeid(*node).name() of the host
// framework's autograd nodes, reads node->getInputs(), and walks node->getUpStreamNodes()
// to assemble fused backward sequences; CTorch's node classes are not part of the reference
// tree, so these carry exactly that: a type, the forward inputs and the upstream links.
#pragma once

#include <memory>
#include <vector>

#include "Tensor.h"

class Node {
 public:
  explicit Node(std::vector<Tensor> inputs = {}) : inputs_(std::move(inputs)) {}
  virtual ~Node() = default;
  const std::vector<Tensor>& getInputs() const { return inputs_; }
  // Nodes that produced this node's inputs (the next step of the backward pass).
  const std::vector<std::shared_ptr<Node>>& getUpStreamNodes() const { return upstream_; }
  void setUpStreamNodes(std::vector<std::shared_ptr<Node>> upstream) { upstream_ = std::move(upstream); }

 private:
  std::vector<Tensor> inputs_;
  std::vector<std::shared_ptr<Node>> upstream_;
};

#define C3_AUTOGRAD_NODE(Name)                                         \
  class Name : public Node {                                           \
   public:                                                             \
    explicit Name(std::vector<Tensor> inputs = {}) : Node(std::move(inputs)) {} \
  };

C3_AUTOGRAD_NODE(ReLUNode)
C3_AUTOGRAD_NODE(SigmoidNode)
C3_AUTOGRAD_NODE(TanhNode)
C3_AUTOGRAD_NODE(AddNode)
C3_AUTOGRAD_NODE(SubNode)
C3_AUTOGRAD_NODE(MulNode)
C3_AUTOGRAD_NODE(DivNode)
C3_AUTOGRAD_NODE(NegNode)
C3_AUTOGRAD_NODE(MatMulNode)
C3_AUTOGRAD_NODE(ExpNode)
C3_AUTOGRAD_NODE(LogNode)
C3_AUTOGRAD_NODE(FactorNode)  // a wrapper node with one upstream (skipped by fused sequences)

#undef C3_AUTOGRAD_NODE
