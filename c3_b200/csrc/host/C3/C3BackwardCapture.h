// Backward capture of the C3 API (the reference's include/C3/C3BackwardCapture.h:62-487 and
// src/C3/C3BackwardCapture.cpp). For every autograd node the host's backward pass visits,
// tryExecuteBackward looks up one single-output kernel per forward input under the key
//   typeid(*node).name() + "|grad:" + dims + ",|inputs:" + dims + ",|in:" + i
// and runs them all, or returns nullopt (the host then runs its own backward) after
// scheduling background compiles of the missing kernels. Backward graphs are built per node
// type as in the reference (ReLU -> Mul(Gt(x,0), grad), MatMul -> grad @ B^T / A^T @ grad with
// the transposes folded into the GEMM operand reads, Add -> identity or SumReduce, and the
// elementwise types), then bound to B200 kernels by C3Engine.
#pragma once

#include <deque>
#include <future>
#include <mutex>
#include <optional>
#include <shared_mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "AutoGrad/Node.h"
#include "C3/C3Engine.h"
#include "C3/C3KernelRegistry.h"
#include "C3/Graph.h"

namespace ct {
namespace c3 {

class C3BackwardCapture {
 public:
  // graph + indices of the forward inputs feeding graph inputs 1.. (input 0 is grad)
  using BackwardGraph = std::pair<Graph, std::vector<size_t>>;

  static C3BackwardCapture& getInstance();

  void clear();
  void clearCallScopedState();

  std::optional<std::vector<Tensor>> tryExecuteBackward(const ::Node* node, const Tensor& grad,
                                                        const std::vector<Tensor>& forward_inputs);
  void compileBackwardAsync(const ::Node* node, const Tensor& grad);
  void compileBackwardAsyncForInput(const ::Node* node, const Tensor& grad, size_t input_index);

  std::optional<Graph> buildBackwardGraph(const ::Node* node, const TensorDesc& grad_desc,
                                          const std::vector<TensorDesc>& input_descs);
  std::optional<Graph> buildBackwardGraphForInput(const ::Node* node, size_t input_index,
                                                  const TensorDesc& grad_desc,
                                                  const std::vector<TensorDesc>& input_descs);
  std::optional<BackwardGraph> buildBackwardGraphForTypeAndIndex(const std::string& node_type,
                                                                 size_t input_index,
                                                                 const TensorDesc& grad_desc,
                                                                 const std::vector<TensorDesc>& input_descs);
  static bool supportsNodeType(const std::string& node_type);

  struct Stats {
    size_t capture_count = 0;
    size_t compile_count = 0;
    size_t cache_hit_count = 0;
    size_t cache_miss_count = 0;
    size_t execution_failures = 0;
    size_t fusion_compile_count = 0;
    size_t fusion_hit_count = 0;
    size_t fusion_miss_count = 0;
  };
  Stats getStats() const;

  // Backward key prefix of a node (without the "|in:i" suffix).
  static std::string makeBaseKey(const std::string& type_name, const std::vector<size_t>& grad_shape,
                                 const std::vector<std::vector<size_t>>& input_shapes);

  // Waits for every background compile (bounded per compile by 30 s).
  void waitForPendingCompiles();

  // ---- fused backward sequences (src/C3/C3BackwardCapture.cpp:874-1637) ----------------
  // The host records every backward node it visits; chains of 2..kFusionWindowSize unary
  // elementwise nodes with one gradient shape are compiled (after kFusionThreshold sightings)
  // into one multi-output kernel, installed under makeFusedBackwardKey. At the chain's most
  // downstream node, tryExecuteFusedBackward walks upstream, runs the kernel once, returns
  // that node's gradient and keeps the others; the upstream nodes then receive theirs from
  // the intercept table (path A) without running anything.
  static constexpr size_t kFusionWindowSize = 4;
  static constexpr int kFusionThreshold = 1;
  void recordBackwardNode(const std::string& node_type, const std::vector<size_t>& grad_shape,
                          const std::vector<size_t>& input_shape, const std::vector<Tensor>& forward_inputs);
  std::optional<Tensor> tryExecuteFusedBackward(const ::Node* node, const Tensor& grad,
                                                const std::vector<Tensor>& forward_inputs);
  static bool isElementWiseBackward(const std::string& node_type);
  static bool isFusableSequence(const std::vector<std::string>& types);
  static std::string makeSequenceKey(const std::vector<std::string>& types);
  static std::string makeFusedBackwardKey(const std::string& seq_key, const std::vector<size_t>& grad_shape,
                                          const std::vector<size_t>& input_shape);
  // Drops intercepted gradients and miss markers (end of a backward pass).
  void clearInterceptedState();

  static bool needsSumReduce(const std::vector<size_t>& grad_shape, const std::vector<size_t>& target_shape);
  static int computeReduceAxis(const std::vector<size_t>& grad_shape, const std::vector<size_t>& target_shape);

 private:
  C3BackwardCapture() = default;
  ~C3BackwardCapture();

  static BackwardGraph buildReLUBackwardGraph(const TensorDesc& grad, const TensorDesc& x);
  static BackwardGraph buildSigmoidBackwardGraph(const TensorDesc& grad, const TensorDesc& x);
  static BackwardGraph buildTanhBackwardGraph(const TensorDesc& grad, const TensorDesc& x);
  static BackwardGraph buildAddBackwardGraph(const TensorDesc& grad, const TensorDesc& lhs,
                                             const TensorDesc& rhs, size_t index);
  static BackwardGraph buildMulBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                             const TensorDesc& b, size_t index);
  static BackwardGraph buildMatMulBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                                const TensorDesc& b, size_t index);
  static BackwardGraph buildNegBackwardGraph(const TensorDesc& grad);
  static BackwardGraph buildSubBackwardGraph(const TensorDesc& grad, size_t index);
  static BackwardGraph buildDivBackwardGraph(const TensorDesc& grad, const TensorDesc& a,
                                             const TensorDesc& b, size_t index);
  static BackwardGraph buildExpBackwardGraph(const TensorDesc& grad, const TensorDesc& x);
  static BackwardGraph buildLogBackwardGraph(const TensorDesc& grad, const TensorDesc& x);

  struct BackwardSequence {
    std::vector<std::string> node_types;
    std::vector<std::vector<size_t>> grad_shapes, input_shapes;
    int frequency = 0;
    bool compiling = false;
  };
  void countSequence(std::vector<std::string> types, std::vector<std::vector<size_t>> gs,
                     std::vector<std::vector<size_t>> is);
  void compileFusedBackwardAsync(const BackwardSequence& seq);

  std::mutex fusion_mutex_;
  std::deque<std::string> recent_sequence_;
  std::deque<std::vector<size_t>> recent_grad_shapes_, recent_input_shapes_;
  std::unordered_map<std::string, BackwardSequence> sequence_counts_;
  std::shared_mutex intercepted_mutex_;
  std::unordered_map<const ::Node*, std::pair<std::string, Tensor>> pending_intercepted_;
  std::mutex miss_marker_mutex_;
  std::unordered_map<const ::Node*, bool> miss_marker_nodes_;
  size_t fusion_compile_count_ = 0, fusion_hit_count_ = 0, fusion_miss_count_ = 0;

  mutable std::mutex stats_mutex_;
  size_t capture_count_ = 0, compile_count_ = 0, cache_hit_count_ = 0, cache_miss_count_ = 0;
  size_t execution_failures_ = 0;
  std::mutex pending_mutex_;
  std::unordered_map<std::string, bool> pending_compiles_;
  std::vector<std::future<void>> futures_;
};

}  // namespace c3
}  // namespace ct
