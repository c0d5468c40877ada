#include "C3/C3KernelRegistry.h"

#include <chrono>

#include "C3/C3Engine.h"
#include "CtorchError.h"

namespace ct {
namespace c3 {

namespace {
std::string shapeToString(const std::vector<size_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

std::string patternOf(const std::vector<op>& seq) {
  std::string p;
  for (size_t i = 0; i < seq.size(); ++i) p += (i ? "+" : "") + std::string(opName(seq[i]));
  return p;
}
}  // namespace

C3KernelRegistry& C3KernelRegistry::getInstance() {
  static C3KernelRegistry instance;
  return instance;
}

size_t C3KernelRegistry::hashShapes(const std::vector<size_t>& lhs, const std::vector<size_t>& rhs) {
  size_t h = 1469598103934665603ull;  // FNV-1a offset basis
  auto mix = [&h](size_t v) {
    h ^= v;
    h *= 1099511628211ull;  // FNV prime
  };
  mix(lhs.size());
  for (auto s : lhs) mix(s);
  mix(rhs.size());
  for (auto s : rhs) mix(s);
  return h;
}

std::string C3KernelRegistry::makeFusedKey(op op_type, const KernelShapeInfo& shapes) {
  std::string key = shapes.fused_pattern;
  key += "|";
  key += std::to_string(static_cast<size_t>(op_type));
  for (auto s : shapes.lhs_shape) key += ":" + std::to_string(s);
  return key;
}

void C3KernelRegistry::install(op op_type, DeviceType dev, std::shared_ptr<CompiledKernel> kernel,
                               const KernelShapeInfo& shapes) {
  if (!kernel) return;
  std::lock_guard<std::mutex> lock(mutex_);
  const auto key = makeKey(op_type, dev, shapes.lhs_shape, shapes.rhs_shape);
  auto it = entries_.find(key);
  if (it != entries_.end() && it->second.active && it->second.kernel &&
      kernel->optLevel() <= it->second.kernel->optLevel())
    return;  // a lower or equal optimisation level never replaces an installed kernel
  entries_[key] = C3Entry{std::move(kernel), shapes, true};
  install_count_.fetch_add(1, std::memory_order_release);
}

void C3KernelRegistry::uninstall(op op_type, DeviceType dev) {
  std::lock_guard<std::mutex> lock(mutex_);
  size_t removed = 0;
  for (auto it = entries_.begin(); it != entries_.end();) {
    if (it->first.first == static_cast<size_t>(op_type) && it->first.second == static_cast<size_t>(dev)) {
      it = entries_.erase(it);
      ++removed;
    } else {
      ++it;
    }
  }
  if (removed) uninstall_count_.fetch_add(removed, std::memory_order_release);
}

void C3KernelRegistry::uninstallAll() {
  std::lock_guard<std::mutex> lock(mutex_);
  uninstall_count_.fetch_add(entries_.size(), std::memory_order_release);
  entries_.clear();
  fused_entries_.clear();
  backward_entries_.clear();
}

bool C3KernelRegistry::validateOutputShape(op op_type, DeviceType dev, const Tensor& out,
                                           const std::vector<size_t>& expected) {
  if (expected.empty() || out.shape() == expected) return true;
  CtorchError::log(ErrorLevel::WARN, ErrorPlatform::kGENERAL, ErrorType::DIMENSION,
                   "[C3-SHAPE-CHECK] op=" + std::to_string(static_cast<int>(op_type)) +
                       " expected=" + shapeToString(expected) + " actual=" + shapeToString(out.shape()) +
                       " — uninstalling defective kernel");
  uninstall(op_type, dev);
  return false;
}

std::optional<Tensor> C3KernelRegistry::tryExecute(op op_type, const Tensor& a, const Tensor& b) {
  C3Entry entry;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = entries_.find(makeKey(op_type, a.device(), a.shape(), b.shape()));
    if (it == entries_.end() || !it->second.active) return std::nullopt;
    entry = it->second;
  }
  if (a.shape() != entry.shapes.lhs_shape || b.shape() != entry.shapes.rhs_shape || !entry.kernel)
    return std::nullopt;
  try {
    const auto t0 = std::chrono::steady_clock::now();
    auto outs = entry.kernel->execute({a, b});
    if (outs.empty()) return std::nullopt;
    recordPerfC3SingleInvoke(static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                                        std::chrono::steady_clock::now() - t0)
                                                        .count()));
    hit_count_.fetch_add(1, std::memory_order_relaxed);
    if (!validateOutputShape(op_type, a.device(), outs[0], entry.shapes.out_shape)) return std::nullopt;
    return outs[0];
  } catch (const std::exception& e) {
    miss_count_.fetch_add(1, std::memory_order_relaxed);
    CtorchError::log(ErrorLevel::DEBUG, ErrorPlatform::kCUDA, ErrorType::RUNTIME,
                     std::string("C3KernelRegistry::tryExecute: ") + e.what());
    return std::nullopt;
  }
}

std::optional<Tensor> C3KernelRegistry::tryExecuteUnary(op op_type, const Tensor& a) {
  C3Entry entry;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = entries_.find(makeKey(op_type, a.device(), a.shape(), {}));
    if (it == entries_.end() || !it->second.active) return std::nullopt;
    entry = it->second;
  }
  if (a.shape() != entry.shapes.lhs_shape || !entry.kernel) return std::nullopt;
  try {
    auto outs = entry.kernel->execute({a});
    if (outs.empty()) return std::nullopt;
    hit_count_.fetch_add(1, std::memory_order_relaxed);
    if (!validateOutputShape(op_type, a.device(), outs[0], entry.shapes.out_shape)) return std::nullopt;
    return outs[0];
  } catch (const std::exception& e) {
    miss_count_.fetch_add(1, std::memory_order_relaxed);
    CtorchError::log(ErrorLevel::DEBUG, ErrorPlatform::kCUDA, ErrorType::RUNTIME,
                     std::string("C3KernelRegistry::tryExecuteUnary: ") + e.what());
    return std::nullopt;
  }
}

C3KernelRegistry::Stats C3KernelRegistry::getStats() const {
  Stats s;
  s.install_count = install_count_.load();
  s.uninstall_count = uninstall_count_.load();
  s.hit_count = hit_count_.load();
  s.miss_count = miss_count_.load();
  s.bypass_count = bypass_count_.load();
  s.fused_hit_count = fused_hit_count_.load();
  s.backward_hit_count = backward_hit_count_.load();
  s.region_dispatch_ns = region_dispatch_ns_.load();
  s.region_match_ns = region_match_ns_.load();
  s.c3_single_invoke_ns = c3_single_invoke_ns_.load();
  s.eager_invoke_ns = eager_invoke_ns_.load();
  s.region_dispatch_count = region_dispatch_count_.load();
  s.region_match_count = region_match_count_.load();
  s.c3_single_invoke_count = c3_single_invoke_count_.load();
  s.eager_invoke_count = eager_invoke_count_.load();
  s.region_cost_rejected_count = region_cost_rejected_count_.load();
  std::lock_guard<std::mutex> lock(mutex_);
  s.active_entries = entries_.size();
  s.fused_entries = fused_entries_.size();
  s.backward_entries = backward_entries_.size();
  return s;
}

void C3KernelRegistry::installFused(std::shared_ptr<CompiledKernel> kernel, op op_type,
                                    const KernelShapeInfo& shapes) {
  if (!kernel) return;
  std::lock_guard<std::mutex> lock(mutex_);
  const std::string key = makeFusedKey(op_type, shapes);
  auto it = fused_entries_.find(key);
  if (it != fused_entries_.end() && it->second.active && it->second.kernel &&
      kernel->optLevel() <= it->second.kernel->optLevel())
    return;
  fused_entries_[key] = FusedEntry{std::move(kernel), shapes, true};
  install_count_.fetch_add(1, std::memory_order_release);
}

std::optional<Tensor> C3KernelRegistry::tryExecuteFused(op op_type, const std::vector<Tensor>& inputs) {
  // Looks up the fused entry whose last op is `op_type` and whose first-op lhs shape matches
  // inputs[0] (the key convention of installFused).
  if (inputs.empty()) return std::nullopt;
  std::shared_ptr<CompiledKernel> kernel;
  KernelShapeInfo shapes;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    for (const auto& [key, e] : fused_entries_) {
      if (!e.active || e.shapes.lhs_shape != inputs[0].shape()) continue;
      if (key != makeFusedKey(op_type, e.shapes)) continue;
      kernel = e.kernel;
      shapes = e.shapes;
      break;
    }
  }
  if (!kernel) return std::nullopt;
  Tensor out = executeFusedWithInputs(kernel, inputs, shapes);
  if (!out.defined()) return std::nullopt;
  return out;
}

Tensor C3KernelRegistry::executeFusedWithInputs(std::shared_ptr<CompiledKernel> kernel,
                                                const std::vector<Tensor>& inputs,
                                                const KernelShapeInfo& shapes) {
  (void)shapes;
  if (!kernel || inputs.empty()) return Tensor();
  try {
    const auto t0 = std::chrono::steady_clock::now();
    auto outs = kernel->execute(inputs);
    recordPerfRegionMatch(static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count()));
    if (outs.empty()) return Tensor();
    fused_hit_count_.fetch_add(1, std::memory_order_relaxed);
    return outs[0];
  } catch (const std::exception& e) {
    CtorchError::log(ErrorLevel::WARN, ErrorPlatform::kGENERAL, ErrorType::UNKNOWN,
                     "C3KernelRegistry::executeFusedWithInputs: kernel execute failed: " +
                         std::string(e.what()) + ", falling back to eager.");
    return Tensor();
  }
}

void C3KernelRegistry::installBackward(const std::string& backward_key, std::shared_ptr<CompiledKernel> kernel,
                                       const std::vector<size_t>& grad_shape,
                                       const std::vector<size_t>& out_shape,
                                       const std::vector<size_t>& fwd_input_map, size_t num_inputs) {
  if (!kernel) return;
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = backward_entries_.find(backward_key);
  if (it != backward_entries_.end() && it->second.active && it->second.kernel &&
      kernel->optLevel() <= it->second.kernel->optLevel())
    return;
  backward_entries_[backward_key] =
      BackwardEntry{std::move(kernel), grad_shape, out_shape, fwd_input_map, num_inputs, true};
  install_count_.fetch_add(1, std::memory_order_release);
}

bool C3KernelRegistry::hasBackwardKey(const std::string& backward_key) const {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = backward_entries_.find(backward_key);
  return it != backward_entries_.end() && it->second.active;
}

std::optional<std::vector<Tensor>> C3KernelRegistry::tryExecuteBackward(
    const std::string& backward_key, const Tensor& grad, const std::vector<Tensor>& forward_inputs) {
  BackwardEntry entry;
  {
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = backward_entries_.find(backward_key);
    if (it == backward_entries_.end() || !it->second.active) return std::nullopt;
    entry = it->second;
  }
  if (grad.shape() != entry.grad_shape) return std::nullopt;
  try {
    // Graph inputs are [grad, forward_inputs[map[0]], forward_inputs[map[1]], ...]
    // (src/C3/C3KernelRegistry.cpp:283-315).
    std::vector<Tensor> inputs;
    inputs.reserve(1 + entry.fwd_input_map.size());
    inputs.push_back(grad);
    for (size_t idx : entry.fwd_input_map) {
      if (idx >= forward_inputs.size()) return std::nullopt;
      inputs.push_back(forward_inputs[idx]);
    }
    if (inputs.size() != entry.num_inputs) return std::nullopt;
    auto outs = entry.kernel->execute(inputs);
    if (outs.empty()) return std::nullopt;
    backward_hit_count_.fetch_add(1, std::memory_order_relaxed);
    return outs;
  } catch (const std::exception& e) {
    CtorchError::log(ErrorLevel::DEBUG, ErrorPlatform::kCUDA, ErrorType::RUNTIME,
                     "C3KernelRegistry::tryExecuteBackward " + backward_key + ": " + e.what());
    return std::nullopt;
  }
}

std::optional<std::pair<std::shared_ptr<CompiledKernel>, KernelShapeInfo>>
C3KernelRegistry::findFusedKernelForSequence(const std::vector<op>& op_seq, DeviceType dev,
                                             const std::vector<size_t>& first_input_shape) {
  (void)dev;
  if (op_seq.empty()) return std::nullopt;
  const std::string pattern = patternOf(op_seq);
  std::lock_guard<std::mutex> lock(mutex_);
  for (const auto& [key, e] : fused_entries_) {
    (void)key;
    if (!e.active || e.shapes.fused_pattern != pattern) continue;
    if (!first_input_shape.empty() && e.shapes.lhs_shape != first_input_shape) continue;
    return std::make_pair(e.kernel, e.shapes);
  }
  return std::nullopt;
}

std::optional<std::pair<std::shared_ptr<CompiledKernel>, KernelShapeInfo>>
C3KernelRegistry::findFusedKernelForFirstOp(op op_type, const std::vector<size_t>& input_shape, DeviceType dev) {
  (void)dev;
  const std::string first = opName(op_type);
  std::lock_guard<std::mutex> lock(mutex_);
  for (const auto& [key, e] : fused_entries_) {
    (void)key;
    if (!e.active || e.shapes.lhs_shape != input_shape) continue;
    const auto& p = e.shapes.fused_pattern;
    if (p.compare(0, first.size(), first) == 0 && (p.size() == first.size() || p[first.size()] == '+'))
      return std::make_pair(e.kernel, e.shapes);
  }
  return std::nullopt;
}

void C3KernelRegistry::uninstallFused(op op_type, const KernelShapeInfo& shapes) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = fused_entries_.find(makeFusedKey(op_type, shapes));
  if (it != fused_entries_.end()) {
    fused_entries_.erase(it);
    uninstall_count_.fetch_add(1, std::memory_order_release);
  }
}

size_t C3KernelRegistry::fusedEntryCount() const {
  std::lock_guard<std::mutex> lock(mutex_);
  return fused_entries_.size();
}

}  // namespace c3
}  // namespace ct
