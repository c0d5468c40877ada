// Hot-path detection and install trigger of the C3 API (the reference's
// include/C3/C3HotPathManager.h:60-1079): per-(op, shape, device) call counting with a
// threshold, cooldown and back-pressure; a 32-entry ring buffer of recent dispatches that is
// matched against the fusion patterns MatMul+Add+{ReLU,Sigmoid} and MatMul+{ReLU,Sigmoid};
// background compile of the matched region through C3Engine (which binds it to the
// precompiled sm_100a kernels) and installation into C3KernelRegistry (fused entry) and
// RegionFusionRegistry (cost-gated, key = rolling hash ^ first-input shape); dual-tier
// single-op compile (opt 2 then opt 4, the higher level wins). Futures are tracked so
// shutdown() can wait for them (30 s bound).
#pragma once

#include <atomic>
#include <chrono>
#include <cstddef>
#include <deque>
#include <future>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "C3/C3Engine.h"
#include "C3/Graph.h"
#include "Ctools.h"

namespace ct {
namespace c3 {

struct HotPathConfig {
  size_t hot_threshold = 5;
  size_t cooldown_sec = 60;
  size_t max_pending = 16;
  uint32_t compile_timeout_ms = 30000;
  bool verbose = false;
};

class C3HotPathManager {
 public:
  static C3HotPathManager& instance();

  void configure(const HotPathConfig& cfg);
  HotPathConfig getConfig() const;

  struct Stats {
    size_t calls_tracked = 0;
    size_t compilations_triggered = 0;
    size_t pending_compiles = 0;
    size_t cooldown_hits = 0;
    size_t backpressure_hits = 0;
  };
  Stats getStats() const;

  struct DispatchRecord {
    op op_type;
    std::vector<size_t> shape;  // lhs ++ rhs (MatMul: {M, K, K, N})
    std::vector<size_t> lhs_shape;
    std::vector<size_t> rhs_shape;
    std::chrono::steady_clock::time_point timestamp;
  };

  void shutdown();
  bool isShuttingDown() const { return shutting_down_.load(std::memory_order_acquire); }
  void waitForPendingCompiles();

  void recordCall(op op_type, DeviceType dev, const std::vector<size_t>& lhs_shape,
                  const std::vector<size_t>& rhs_shape = {}, bool in_autograd = false);
  void clear();

  static Graph buildFusedGraphForTest(const std::vector<DispatchRecord>& records, const std::string& pattern) {
    return buildFusedGraph(records, pattern);
  }

 private:
  C3HotPathManager() = default;
  ~C3HotPathManager();
  C3HotPathManager(const C3HotPathManager&) = delete;
  C3HotPathManager& operator=(const C3HotPathManager&) = delete;

  struct HotEntry {
    size_t call_count = 0;
    bool compiling = false;
    std::chrono::steady_clock::time_point last_compile_time;
  };
  static constexpr size_t kMaxRingBufferSize = 32;

  static size_t hashShapeKey(const std::vector<size_t>& shape, op op_type, DeviceType dev);
  static Graph buildGraphForOp(op op_type, const std::vector<size_t>& shape, const std::vector<size_t>& lhs,
                               const std::vector<size_t>& rhs);
  static Graph buildFusedGraph(const std::vector<DispatchRecord>& records, const std::string& pattern);
  static bool isSupportedOp(op o);
  static bool isUnaryOp(op o);
  static std::vector<size_t> extractBinOpOutShape(const std::vector<size_t>& shape);

  void tryFuseRecentDispatches(DeviceType dev, const HotPathConfig& cfg);
  void submitFusedCompileAsync(const std::vector<DispatchRecord>& records, DeviceType dev,
                               const HotPathConfig& cfg, const std::string& pattern);
  void submitCompileAsync(op op_type, DeviceType dev, const std::vector<size_t>& shape,
                          const std::vector<size_t>& lhs, const std::vector<size_t>& rhs, size_t key,
                          const HotPathConfig& cfg);
  void track(std::future<void> f);

  mutable std::mutex mutex_, cfg_mutex_, rb_mutex_, futures_mutex_;
  HotPathConfig config_;
  std::unordered_map<size_t, HotEntry> entries_;
  std::deque<DispatchRecord> recent_dispatches_;
  std::vector<std::future<void>> pending_futures_;
  std::atomic<size_t> calls_tracked_{0}, compilations_triggered_{0}, pending_compiles_{0};
  std::atomic<bool> shutting_down_{false};
  size_t cooldown_hits_ = 0, backpressure_hits_ = 0;
};

}  // namespace c3
}  // namespace ct
