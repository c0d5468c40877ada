// Compile engine of the C3 API (the reference's include/C3/C3Engine.h:45-640), B200 build.
//
// CompiledKernel keeps the reference's virtual interface (execute / cacheKey / targetDevice /
// workspaceBytes / outShape / installIntoRegistry / optLevel) and its error contract: execute
// throws std::runtime_error on failure and callers (the registries) turn that into nullopt.
// C3Engine::compile no longer generates code: it matches the graph against the regions the
// B200 kernels implement (C3/CudaKernels.h) and returns a kernel object bound to them. The
// cache (LRU, 256 entries, keyed by graph text + options), async compile with de-duplication
// and a watchdog timeout, error recording and shutdown follow the reference's semantics.
#pragma once

#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <future>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "C3/C3KernelRegistry.h"
#include "C3/Graph.h"
#include "Ctools.h"
#include "Tensor.h"

namespace ct {
namespace c3 {

struct EngineState;

enum class C3Backend { Handwritten = 0, MLIR = 1, CUDA = 2 };

// Arithmetic the CUDA kernels use for fp32 tensors. bf16 tensors always take the tcgen05
// tensor-core path (fp32 accumulation).
enum class Precision {
  kExactF32 = 0,  // CUDA-core kernels reproducing the reference's fp32 loops bit for bit
  kBF16 = 1,      // round fp32 operands to bf16 and use the tensor cores
};

struct CompileOptions {
  C3Backend backend = C3Backend::CUDA;
  DeviceType target_device = DeviceType::kCUDA;
  int opt_level = 3;
  bool enable_fusion = true;
  bool enable_cache = true;
  bool enable_autotune = false;
  bool enable_profiling = false;
  bool pgo_mode = false;
  Precision fp32_precision = Precision::kExactF32;
  std::string cache_key_override;
};

struct C3CacheStats {
  size_t total_entries = 0;
  size_t hits = 0;
  size_t misses = 0;
  size_t evictions = 0;
  size_t bytes_used = 0;
  size_t pending_compiles = 0;
  size_t async_completions = 0;
  size_t async_failures = 0;
};

struct ProfileData {
  std::atomic<uint64_t> call_count{0};
  std::atomic<uint64_t> total_time_ns{0};
  std::atomic<uint64_t> min_time_ns{UINT64_MAX};
  std::atomic<uint64_t> max_time_ns{0};
  std::atomic<uint64_t> last_time_ns{0};

  void record(uint64_t ns) {
    call_count.fetch_add(1, std::memory_order_relaxed);
    total_time_ns.fetch_add(ns, std::memory_order_relaxed);
    last_time_ns.store(ns, std::memory_order_relaxed);
    uint64_t lo = min_time_ns.load(std::memory_order_relaxed);
    while (ns < lo && !min_time_ns.compare_exchange_weak(lo, ns, std::memory_order_relaxed)) {}
    uint64_t hi = max_time_ns.load(std::memory_order_relaxed);
    while (ns > hi && !max_time_ns.compare_exchange_weak(hi, ns, std::memory_order_relaxed)) {}
  }
  uint64_t avgTimeNs() const {
    const uint64_t c = call_count.load(std::memory_order_relaxed);
    return c ? total_time_ns.load(std::memory_order_relaxed) / c : 0;
  }
};

class CompiledKernel {
 public:
  virtual ~CompiledKernel() = default;
  // Inputs in graph-input order; outputs in graph-output order (a kernel may append extra
  // outputs after them, e.g. the region kernel's ReLU bit mask). Throws on failure.
  virtual std::vector<Tensor> execute(const std::vector<Tensor>& inputs) = 0;
  virtual const std::string& cacheKey() const = 0;
  virtual DeviceType targetDevice() const = 0;
  virtual size_t workspaceBytes() const = 0;
  virtual std::optional<std::vector<size_t>> outShape() const { return std::nullopt; }
  virtual bool installIntoRegistry(op op_type, const KernelShapeInfo& shapes);
  virtual int optLevel() const { return opt_level_; }
  void setOptLevel(int level) { opt_level_ = level; }

 protected:
  int opt_level_ = 3;
};

// Times every execute() (host wall clock, including the device work it waits for).
class ProfiledCompiledKernel : public CompiledKernel {
 public:
  ProfiledCompiledKernel(std::shared_ptr<CompiledKernel> inner, std::shared_ptr<ProfileData> data)
      : inner_(std::move(inner)), data_(std::move(data)) {}
  std::vector<Tensor> execute(const std::vector<Tensor>& inputs) override {
    const auto t0 = std::chrono::steady_clock::now();
    auto out = inner_->execute(inputs);
    const auto t1 = std::chrono::steady_clock::now();
    data_->record(static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count()));
    return out;
  }
  const std::string& cacheKey() const override { return inner_->cacheKey(); }
  DeviceType targetDevice() const override { return inner_->targetDevice(); }
  size_t workspaceBytes() const override { return inner_->workspaceBytes(); }
  std::optional<std::vector<size_t>> outShape() const override { return inner_->outShape(); }
  bool installIntoRegistry(op o, const KernelShapeInfo& s) override {
    return inner_->installIntoRegistry(o, s);
  }
  int optLevel() const override { return inner_->optLevel(); }
  CompiledKernel& inner() { return *inner_; }
  const ProfileData& profileData() const { return *data_; }

 private:
  std::shared_ptr<CompiledKernel> inner_;
  std::shared_ptr<ProfileData> data_;
};

using CompileFuture = std::shared_future<std::shared_ptr<CompiledKernel>>;

class C3Engine {
 public:
  static C3Engine& getInstance();

  // Maps `graph` onto the B200 kernels. Throws std::runtime_error when no kernel implements it.
  std::shared_ptr<CompiledKernel> compile(const Graph& graph, const CompileOptions& options = {});
  // Non-blocking; identical pending requests share one future; the future yields nullptr on
  // failure or when the watchdog timeout passes first.
  CompileFuture compileAsync(const Graph& graph, const CompileOptions& options = {});
  std::vector<std::shared_ptr<CompiledKernel>> compileParallel(const std::vector<Graph>& graphs,
                                                               const CompileOptions& options = {});
  // Compiles and installs single-op graphs (MatMul / elementwise) into C3KernelRegistry.
  std::shared_ptr<CompiledKernel> compileAndInject(const Graph& graph, const CompileOptions& options = {});

  std::shared_ptr<CompiledKernel> getKernel(const std::string& cache_key) const;
  C3CacheStats getCacheStats() const;
  std::shared_ptr<ProfileData> getProfileData(const std::string& cache_key) const;
  std::string getLastCompileError() const;
  void clearLastCompileError();
  void recordCompileError(const std::string& prefix, const std::string& err);
  bool wasAsyncCompileTimedOut(const std::string& cache_key) const;
  void setCompileTimeoutMs(uint32_t ms);
  uint32_t getCompileTimeoutMs() const;
  void clearCache();
  void shutdown();

  // Cache key of a graph under options (exposed for tests and the async-timeout query).
  static std::string makeCacheKey(const Graph& graph, const CompileOptions& options);

  static EngineState& getState();

 private:
  C3Engine();
  ~C3Engine();
  C3Engine(const C3Engine&) = delete;
  C3Engine& operator=(const C3Engine&) = delete;
  std::shared_ptr<CompiledKernel> doCompile(const Graph& graph, const CompileOptions& options,
                                            const std::string& key);
  std::unique_ptr<EngineState> state_;
};

}  // namespace c3
}  // namespace ct
