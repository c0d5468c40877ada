#include "C3/RegionFusion.h"

namespace ct {
namespace c3 {

RegionFusionRegistry& RegionFusionRegistry::getInstance() {
  static RegionFusionRegistry instance;
  RollingHash::precompute(256);
  return instance;
}

// Caller holds mutex_.
void RegionFusionRegistry::publish(uint64_t hash, RegionEntry&& e) {
  storage_.push_back(std::make_unique<RegionEntry>(std::move(e)));
  entries_[hash] = storage_.back().get();
}

void RegionFusionRegistry::markLastOp(const std::vector<op>& op_seq) {
  if (!op_seq.empty())
    installed_last_ops_.fetch_or(uint64_t(1) << static_cast<size_t>(op_seq.back()), std::memory_order_release);
  installed_count_.fetch_add(1, std::memory_order_release);
}

void RegionFusionRegistry::install(uint64_t hash, const std::vector<op>& op_seq,
                                   std::shared_ptr<CompiledKernel> kernel,
                                   const std::vector<size_t>& input_shapes) {
  std::lock_guard<std::mutex> lock(mutex_);
  RegionEntry e;
  e.hash = hash;
  e.op_seq = op_seq;
  e.kernel = std::move(kernel);
  e.input_shapes = input_shapes;
  e.num_external_inputs = input_shapes.empty() ? 0 : 1;
  e.len = op_seq.size();
  e.active = true;
  publish(hash, std::move(e));
  markLastOp(op_seq);
}

void RegionFusionRegistry::installFromCompiledKernel(const std::vector<op>& op_seq,
                                                     std::shared_ptr<CompiledKernel> kernel) {
  if (op_seq.empty()) return;
  install(RollingHash::hashSequence(op_seq), op_seq, std::move(kernel), {});
}

uint64_t RegionFusionRegistry::regionKey(const std::vector<op>& op_seq,
                                         const std::vector<std::vector<size_t>>& first_input_shapes) {
  const uint64_t op_hash = RollingHash::hashSequence(op_seq);
  uint64_t shape_hash = 0;
  if (!first_input_shapes.empty())
    for (auto s : first_input_shapes.front()) shape_hash = shape_hash * 31 + s + 1;
  return op_hash ^ (shape_hash << 32);
}

void RegionFusionRegistry::installWithCost(const std::vector<op>& op_seq, std::shared_ptr<CompiledKernel> kernel,
                                           const std::vector<size_t>& out_numels,
                                           const std::vector<std::vector<size_t>>& first_input_shapes) {
  if (op_seq.empty() || !kernel) return;
  const FusionCost cost = FusionCostModel::estimate(op_seq, out_numels);
  const uint64_t hash = regionKey(op_seq, first_input_shapes);
  std::lock_guard<std::mutex> lock(mutex_);
  RegionEntry e;
  e.hash = hash;
  e.op_seq = op_seq;
  e.kernel = std::move(kernel);
  e.len = op_seq.size();
  e.cost = cost;
  e.first_input_shapes = first_input_shapes;
  // active only with complete numels and a worthwhile cost estimate; the last-op mask is set
  // regardless (it is only a fast filter).
  e.active = (out_numels.size() == op_seq.size()) && cost.worthwhile;
  publish(hash, std::move(e));
  markLastOp(op_seq);
}

RegionEntry* RegionFusionRegistry::find(uint64_t hash) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = entries_.find(hash);
  return (it != entries_.end() && it->second->active) ? it->second : nullptr;
}

RegionEntry* RegionFusionRegistry::matchFromPosition(const std::vector<uint64_t>& prefix_hashes,
                                                     size_t current_pos,
                                                     const std::vector<size_t>& /*input_shapes*/) {
  if (prefix_hashes.empty() || current_pos >= prefix_hashes.size() - 1) return nullptr;
  std::lock_guard<std::mutex> lock(mutex_);
  size_t max_len = prefix_hashes.size() - 1 - current_pos;
  if (max_len > 32) max_len = 32;
  for (size_t len = max_len; len >= 2; --len) {
    const uint64_t h = RollingHash::getSubHash(prefix_hashes, current_pos, current_pos + len - 1);
    auto it = entries_.find(h);
    if (it != entries_.end() && it->second->active && it->second->len == len) return it->second;
  }
  return nullptr;
}

size_t RegionFusionRegistry::entryCount() const {
  std::lock_guard<std::mutex> lock(mutex_);
  return entries_.size();
}

bool RegionFusionRegistry::mayMatchAsLastOp(op last_op) const {
  return (installed_last_ops_.load(std::memory_order_acquire) &
          (uint64_t(1) << static_cast<size_t>(last_op))) != 0;
}

void RegionFusionRegistry::clear() {
  std::lock_guard<std::mutex> lock(mutex_);
  entries_.clear();
  storage_.clear();
  installed_last_ops_.store(0, std::memory_order_release);
  installed_count_.store(0, std::memory_order_release);
}

void RegionFusionRegistry::uninstallAll() { clear(); }

}  // namespace c3
}  // namespace ct
