// Region-fusion registry (the reference's include/C3/RegionFusion.h:29-131 and
// src/C3/RegionFusionRegistry.cpp): region kernels keyed by the rolling hash of their op
// sequence, with installWithCost mixing the first input shape into the key
// (key = op_hash ^ (shape_hash << 32), shape_hash = fold(s -> h * 31 + s + 1)) and gating
// activation on the fusion cost model; lock-free installed-count and last-op bitmask
// short-circuits; longest-first matching (<= 32 ops) over unmixed sub-hashes.
#pragma once

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "C3/C3Engine.h"
#include "C3/C3KernelRegistry.h"
#include "C3/FusionCostModel.h"
#include "C3/RollingHash.h"
#include "Ctools.h"
#include "Tensor.h"

namespace ct {
namespace c3 {

struct RegionEntry {
  uint64_t hash = 0;
  std::vector<op> op_seq;
  std::vector<size_t> input_shapes;
  std::vector<std::vector<size_t>> first_input_shapes;
  std::shared_ptr<CompiledKernel> kernel;
  FusedKernelFunc fused_func_ptr = nullptr;
  size_t num_external_inputs = 0;
  size_t len = 0;
  bool active = false;
  FusionCost cost;
};

class RegionFusionRegistry {
 public:
  static RegionFusionRegistry& getInstance();

  void install(uint64_t hash, const std::vector<op>& op_seq, std::shared_ptr<CompiledKernel> kernel,
               const std::vector<size_t>& input_shapes);
  void installFromCompiledKernel(const std::vector<op>& op_seq, std::shared_ptr<CompiledKernel> kernel);
  void installWithCost(const std::vector<op>& op_seq, std::shared_ptr<CompiledKernel> kernel,
                       const std::vector<size_t>& out_numels,
                       const std::vector<std::vector<size_t>>& first_input_shapes = {});

  // Entry for `hash` when active. The entry is immutable and the pointer stays valid until
  // clear()/uninstallAll(), even if the key is reinstalled meanwhile.
  RegionEntry* find(uint64_t hash);
  RegionEntry* matchFromPosition(const std::vector<uint64_t>& prefix_hashes, size_t current_pos,
                                 const std::vector<size_t>& input_shapes);

  size_t entryCount() const;
  size_t installedCountNoLock() const { return installed_count_.load(std::memory_order_acquire); }
  bool mayMatchAsLastOp(op last_op) const;
  void clear();
  void uninstallAll();

  // The key installWithCost files a region under (what a host dispatcher passes to find()).
  static uint64_t regionKey(const std::vector<op>& op_seq, const std::vector<std::vector<size_t>>& first_input_shapes);

 private:
  RegionFusionRegistry() = default;
  RegionFusionRegistry(const RegionFusionRegistry&) = delete;
  RegionFusionRegistry& operator=(const RegionFusionRegistry&) = delete;

  void markLastOp(const std::vector<op>& op_seq);
  void publish(uint64_t hash, RegionEntry&& e);

  mutable std::mutex mutex_;
  // Published entries are immutable: a reinstall under the same key publishes a new entry and
  // the superseded one stays in `storage_` until clear(), so a pointer find() returned is never
  // written while a dispatcher reads it (e.g. the tuned tier replacing the precompiled one).
  std::unordered_map<uint64_t, RegionEntry*> entries_;
  std::vector<std::unique_ptr<RegionEntry>> storage_;
  std::atomic<size_t> installed_count_{0};
  static_assert(static_cast<size_t>(op::kCount) <= 64, "op::kCount exceeds the bitmask");
  std::atomic<uint64_t> installed_last_ops_{0};
};

}  // namespace c3
}  // namespace ct
