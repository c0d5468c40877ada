// Autograd node shim. C3BackwardCapture keys its kernels by typeid(*node).name() of the host
// framework's autograd nodes and reads node->getInputs(); CTorch's node classes are not
// part of the reference tree, so these carry exactly that: a type and the forward inputs.
#pragma once

#include <vector>

#include "Tensor.h"

class Node {
 public:
  explicit Node(std::vector<Tensor> inputs = {}) : inputs_(std::move(inputs)) {}
  virtual ~Node() = default;
  const std::vector<Tensor>& getInputs() const { return inputs_; }

 private:
  std::vector<Tensor> inputs_;
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

#undef C3_AUTOGRAD_NODE
