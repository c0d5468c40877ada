// Thread-safe kernel registry of the C3 API (the reference's include/C3/C3KernelRegistry.h:106-585
// and src/C3/C3KernelRegistry.cpp): single-op entries keyed by (op, device, FNV-1a of the
// input shapes), fused entries keyed by "pattern|op:lhs...", backward entries keyed by the
// C3BackwardCapture string key. Install keeps the higher optLevel (an equal or lower level
// does not replace an active entry); every execution path turns a thrown error into nullopt
// so the caller falls back to its own path; wrong output shapes uninstall the kernel.
#pragma once

#include <atomic>
#include <cstddef>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "Ctools.h"
#include "Tensor.h"

namespace ct {
namespace c3 {

class CompiledKernel;

using C3KernelFunc = void (*)(const float*, const float*, float*, size_t, size_t, size_t, size_t);
using FusedKernelFunc = void (*)(const float* const*, float*, size_t);
using MultiNodeKernelFunc = void (*)(const float* const*, float*, size_t, size_t, size_t, size_t, float*);

struct KernelShapeInfo {
  std::vector<size_t> lhs_shape;
  std::vector<size_t> rhs_shape;
  std::vector<size_t> out_shape;
  bool is_matmul = false;
  size_t M = 0, K = 0, N = 0;
  std::string fused_pattern;
};

class C3KernelRegistry {
 public:
  static C3KernelRegistry& getInstance();

  void install(op op_type, DeviceType dev, std::shared_ptr<CompiledKernel> kernel,
               const KernelShapeInfo& shapes);
  void uninstall(op op_type, DeviceType dev);
  void uninstallAll();

  std::optional<Tensor> tryExecute(op op_type, const Tensor& a, const Tensor& b);
  std::optional<Tensor> tryExecuteUnary(op op_type, const Tensor& a);

  struct Stats {
    size_t install_count = 0;
    size_t uninstall_count = 0;
    size_t hit_count = 0;
    size_t miss_count = 0;
    size_t bypass_count = 0;
    size_t active_entries = 0;
    size_t fused_entries = 0;
    size_t backward_entries = 0;
    size_t fused_hit_count = 0;
    uint64_t region_dispatch_ns = 0;
    uint64_t region_match_ns = 0;
    uint64_t c3_single_invoke_ns = 0;
    uint64_t eager_invoke_ns = 0;
    uint64_t region_dispatch_count = 0;
    uint64_t region_match_count = 0;
    uint64_t c3_single_invoke_count = 0;
    uint64_t eager_invoke_count = 0;
    uint64_t region_cost_rejected_count = 0;
    size_t backward_hit_count = 0;
  };
  Stats getStats() const;
  void recordBypass() { bypass_count_.fetch_add(1, std::memory_order_relaxed); }
  void recordPerfRegionDispatch(uint64_t ns) { add(region_dispatch_ns_, region_dispatch_count_, ns); }
  void recordPerfRegionMatch(uint64_t ns) { add(region_match_ns_, region_match_count_, ns); }
  void recordPerfC3SingleInvoke(uint64_t ns) { add(c3_single_invoke_ns_, c3_single_invoke_count_, ns); }
  void recordPerfEagerInvoke(uint64_t ns) { add(eager_invoke_ns_, eager_invoke_count_, ns); }
  void recordPerfRegionCostRejected() { region_cost_rejected_count_.fetch_add(1, std::memory_order_relaxed); }

  void installFused(std::shared_ptr<CompiledKernel> kernel, op op_type, const KernelShapeInfo& shapes);
  std::optional<Tensor> tryExecuteFused(op op_type, const std::vector<Tensor>& inputs);

  void installBackward(const std::string& backward_key, std::shared_ptr<CompiledKernel> kernel,
                       const std::vector<size_t>& grad_shape, const std::vector<size_t>& out_shape,
                       const std::vector<size_t>& fwd_input_map, size_t num_inputs = 1);
  std::optional<std::vector<Tensor>> tryExecuteBackward(const std::string& backward_key,
                                                        const Tensor& grad,
                                                        const std::vector<Tensor>& forward_inputs = {});
  bool hasBackwardKey(const std::string& backward_key) const;

  std::optional<std::pair<std::shared_ptr<CompiledKernel>, KernelShapeInfo>> findFusedKernelForSequence(
      const std::vector<op>& op_seq, DeviceType dev, const std::vector<size_t>& first_input_shape = {});
  std::optional<std::pair<std::shared_ptr<CompiledKernel>, KernelShapeInfo>> findFusedKernelForFirstOp(
      op op_type, const std::vector<size_t>& input_shape, DeviceType dev);

  // Runs a fused kernel on its raw inputs; returns an undefined Tensor on failure.
  Tensor executeFusedWithInputs(std::shared_ptr<CompiledKernel> kernel, const std::vector<Tensor>& inputs,
                                const KernelShapeInfo& shapes);

  void uninstallFused(op op_type, const KernelShapeInfo& shapes);
  size_t fusedEntryCount() const;

  // Key helpers (exposed for tests: the keys must match what a C3 host computes).
  static size_t hashShapes(const std::vector<size_t>& lhs, const std::vector<size_t>& rhs);
  static std::string makeFusedKey(op op_type, const KernelShapeInfo& shapes);

 private:
  C3KernelRegistry() = default;
  static void add(std::atomic<uint64_t>& ns, std::atomic<uint64_t>& cnt, uint64_t v) {
    ns.fetch_add(v, std::memory_order_relaxed);
    cnt.fetch_add(1, std::memory_order_relaxed);
  }

  struct C3Entry {
    std::shared_ptr<CompiledKernel> kernel;
    KernelShapeInfo shapes;
    bool active = false;
  };
  struct FusedEntry {
    std::shared_ptr<CompiledKernel> kernel;
    KernelShapeInfo shapes;
    bool active = false;
  };
  struct BackwardEntry {
    std::shared_ptr<CompiledKernel> kernel;
    std::vector<size_t> grad_shape;
    std::vector<size_t> out_shape;
    std::vector<size_t> fwd_input_map;
    size_t num_inputs = 1;
    bool active = false;
  };
  struct KeyType {
    size_t first, second, third;
    bool operator==(const KeyType& o) const {
      return first == o.first && second == o.second && third == o.third;
    }
  };
  struct KeyHash {
    size_t operator()(const KeyType& k) const {
      size_t h = k.first;
      h ^= (k.second << 16) + 0x9e3779b9 + (h << 6) + (h >> 2);
      h ^= (k.third << 24) + 0x9e3779b9 + (h << 6) + (h >> 2);
      return h;
    }
  };
  static KeyType makeKey(op o, DeviceType dev, const std::vector<size_t>& lhs, const std::vector<size_t>& rhs) {
    return {static_cast<size_t>(o), static_cast<size_t>(dev), hashShapes(lhs, rhs)};
  }
  bool validateOutputShape(op op_type, DeviceType dev, const Tensor& out,
                           const std::vector<size_t>& expected);

  mutable std::mutex mutex_;
  std::unordered_map<KeyType, C3Entry, KeyHash> entries_;
  std::unordered_map<std::string, FusedEntry> fused_entries_;
  std::unordered_map<std::string, BackwardEntry> backward_entries_;

  std::atomic<size_t> install_count_{0}, uninstall_count_{0}, hit_count_{0}, miss_count_{0};
  std::atomic<size_t> bypass_count_{0}, fused_hit_count_{0}, backward_hit_count_{0};
  std::atomic<uint64_t> region_dispatch_ns_{0}, region_match_ns_{0}, c3_single_invoke_ns_{0},
      eager_invoke_ns_{0}, region_dispatch_count_{0}, region_match_count_{0},
      c3_single_invoke_count_{0}, eager_invoke_count_{0}, region_cost_rejected_count_{0};
};

}  // namespace c3
}  // namespace ct
