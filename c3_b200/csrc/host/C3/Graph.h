// Computation-graph IR of the C3 API (the reference's include/C3/Graph.h:41-450): tensor
// descriptors, the node-variant set, and a Graph with the same building API
// (addInput / addNode / addConstant / markOutput) and accessors. It describes what a region
// computes; C3Engine::compile maps a graph onto the precompiled sm_100a kernels.
#pragma once

#include <cstddef>
#include <string>
#include <variant>
#include <vector>

#include "Ctools.h"

namespace ct {
namespace c3 {

struct TensorDesc {
  std::vector<size_t> shape;
  DType dtype = DType::kFloat;
  DeviceType device = DeviceType::kCPU;
  size_t numel = 0;

  static size_t computeNumel(const std::vector<size_t>& s) {
    size_t n = 1;
    for (size_t d : s) n *= d;
    return n;
  }
  static TensorDesc fromShape(const std::vector<size_t>& s, DType dt = DType::kFloat,
                              DeviceType dev = DeviceType::kCPU) {
    return {s, dt, dev, computeNumel(s)};
  }
  bool operator==(const TensorDesc& o) const {
    return shape == o.shape && dtype == o.dtype && device == o.device;
  }
};

struct AddNode { static constexpr const char* name = "Add"; TensorDesc lhs_desc, rhs_desc; };
struct MulNode { static constexpr const char* name = "Mul"; TensorDesc lhs_desc, rhs_desc; };
struct SubNode { static constexpr const char* name = "Sub"; TensorDesc lhs_desc, rhs_desc; };
struct DivNode { static constexpr const char* name = "Div"; TensorDesc lhs_desc, rhs_desc; };
struct MatMulNode { static constexpr const char* name = "MatMul"; TensorDesc lhs_desc, rhs_desc; };
struct NegNode { static constexpr const char* name = "Neg"; TensorDesc in_desc; };
struct ReLUNode { static constexpr const char* name = "ReLU"; TensorDesc in_desc; };
struct SigmoidNode { static constexpr const char* name = "Sigmoid"; TensorDesc in_desc; };
struct TanhNode { static constexpr const char* name = "Tanh"; TensorDesc in_desc; };
struct GtNode { static constexpr const char* name = "Gt"; TensorDesc lhs_desc, rhs_desc; };
struct SumReduceNode { static constexpr const char* name = "SumReduce"; TensorDesc in_desc; int axis = -1; };
struct TransposeNode { static constexpr const char* name = "Transpose"; TensorDesc in_desc; int dim0 = 0; int dim1 = 1; };
struct ExpNode { static constexpr const char* name = "Exp"; TensorDesc in_desc; };
struct LogNode { static constexpr const char* name = "Log"; TensorDesc in_desc; };
struct ConstNode { static constexpr const char* name = "Const"; double value = 0.0; };

using NodeVariant = std::variant<AddNode, SubNode, MulNode, DivNode, MatMulNode, NegNode, ReLUNode,
                                 SigmoidNode, TanhNode, GtNode, SumReduceNode, TransposeNode,
                                 ExpNode, LogNode, ConstNode>;

const char* nodeName(const NodeVariant& v);

struct Node {
  size_t id = 0;
  NodeVariant op;
  std::vector<size_t> inputs;
  std::vector<size_t> outputs;  // consumers
  TensorDesc out_desc;
};

class Graph {
 public:
  Graph() = default;

  size_t addInput(const TensorDesc& desc);
  size_t addNode(NodeVariant op, const std::vector<size_t>& input_ids, const TensorDesc& out_desc);
  size_t addConstant(double value, const TensorDesc& desc);
  void markOutput(size_t node_id);

  const std::vector<size_t>& inputs() const { return inputs_; }
  const std::vector<size_t>& outputs() const { return outputs_; }
  const std::vector<Node>& nodes() const { return nodes_; }
  const Node& node(size_t id) const { return nodes_[id]; }
  size_t nodeCount() const { return nodes_.size(); }
  size_t inputCount() const { return inputs_.size(); }
  size_t outputCount() const { return outputs_.size(); }
  bool validNodeId(size_t id) const { return id < nodes_.size(); }
  bool isInput(size_t id) const;
  bool isConst(size_t id) const;
  bool isValid() const;

  // Nodes that compute (neither graph inputs nor constants), in insertion (topological) order.
  std::vector<size_t> computeNodes() const;

  // Drops compute nodes that no output depends on.
  Graph eliminateDeadCode() const;

  // Canonical text of the graph; also the compile-cache key component.
  std::string toString() const;

 private:
  std::vector<Node> nodes_;
  std::vector<size_t> inputs_;
  std::vector<size_t> outputs_;
};

}  // namespace c3
}  // namespace ct
