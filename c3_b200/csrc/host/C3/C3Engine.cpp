#include "C3/C3Engine.h"

#include <list>
#include <mutex>
#include <sstream>
#include <unordered_map>

#include "C3/C3KernelRegistry.h"
#include "C3/CudaKernels.h"
#include "CtorchError.h"

namespace ct {
namespace c3 {

struct EngineState {
  mutable std::mutex mu;
  // LRU compile cache: most recently used at the front
  std::list<std::pair<std::string, std::shared_ptr<CompiledKernel>>> lru;
  std::unordered_map<std::string, decltype(lru)::iterator> index;
  std::unordered_map<std::string, std::shared_ptr<ProfileData>> profiles;
  std::unordered_map<std::string, CompileFuture> pending;
  std::vector<std::future<void>> watchers;
  size_t hits = 0, misses = 0, evictions = 0, async_completions = 0, async_failures = 0;
  std::string last_error;
  uint32_t timeout_ms = 30000;
  static constexpr size_t kCapacity = 256;
};

C3Engine::C3Engine() : state_(std::make_unique<EngineState>()) {}
C3Engine::~C3Engine() { shutdown(); }

C3Engine& C3Engine::getInstance() {
  static C3Engine instance;
  return instance;
}

EngineState& C3Engine::getState() { return *getInstance().state_; }

bool CompiledKernel::installIntoRegistry(op op_type, const KernelShapeInfo& shapes) {
  // Shared ownership is required by the registry; kernels created by C3Engine are always
  // held by a shared_ptr, so install a non-owning alias guarded by the engine cache.
  auto self = C3Engine::getInstance().getKernel(cacheKey());
  if (!self || self.get() != this) return false;
  C3KernelRegistry::getInstance().install(op_type, DeviceType::kCUDA, self, shapes);
  C3KernelRegistry::getInstance().install(op_type, DeviceType::kCPU, self, shapes);
  return true;
}

std::string C3Engine::makeCacheKey(const Graph& graph, const CompileOptions& o) {
  if (!o.cache_key_override.empty()) return o.cache_key_override;
  std::ostringstream ss;
  ss << "c3cu|b" << static_cast<int>(o.backend) << "|o" << o.opt_level << "|p"
     << static_cast<int>(o.fp32_precision) << "|prof" << o.enable_profiling << "|" << graph.toString();
  return ss.str();
}

std::shared_ptr<CompiledKernel> C3Engine::doCompile(const Graph& graph, const CompileOptions& options,
                                                    const std::string& key) {
  std::shared_ptr<CompiledKernel> k = lowerGraph(graph, options, key);
  k->setOptLevel(options.opt_level);
  if (options.enable_profiling) {
    auto data = std::make_shared<ProfileData>();
    {
      std::lock_guard<std::mutex> lock(state_->mu);
      state_->profiles[key] = data;
    }
    k = std::make_shared<ProfiledCompiledKernel>(k, data);
  }
  return k;
}

std::shared_ptr<CompiledKernel> C3Engine::compile(const Graph& graph, const CompileOptions& options) {
  const std::string key = makeCacheKey(graph, options);
  if (options.enable_cache) {
    std::lock_guard<std::mutex> lock(state_->mu);
    auto it = state_->index.find(key);
    if (it != state_->index.end()) {
      state_->lru.splice(state_->lru.begin(), state_->lru, it->second);
      ++state_->hits;
      return it->second->second;
    }
    ++state_->misses;
  }
  std::shared_ptr<CompiledKernel> k;
  try {
    k = doCompile(graph, options, key);
  } catch (const std::exception& e) {
    recordCompileError("", e.what());
    throw;
  }
  if (options.enable_cache) {
    std::lock_guard<std::mutex> lock(state_->mu);
    auto it = state_->index.find(key);
    if (it != state_->index.end()) return it->second->second;  // a concurrent compile won
    state_->lru.emplace_front(key, k);
    state_->index[key] = state_->lru.begin();
    while (state_->lru.size() > EngineState::kCapacity) {
      state_->index.erase(state_->lru.back().first);
      state_->lru.pop_back();
      ++state_->evictions;
    }
  }
  return k;
}

CompileFuture C3Engine::compileAsync(const Graph& graph, const CompileOptions& options) {
  const std::string key = makeCacheKey(graph, options);
  std::lock_guard<std::mutex> lock(state_->mu);
  auto pit = state_->pending.find(key);
  if (pit != state_->pending.end()) return pit->second;  // de-duplicated
  const uint32_t timeout_ms = state_->timeout_ms;
  // The compile itself runs to completion even after the watchdog gave up (its result then
  // lands in the cache for the next request), as in the reference.
  auto work = std::async(std::launch::async, [this, graph, options]() -> std::shared_ptr<CompiledKernel> {
                try {
                  return compile(graph, options);
                } catch (const std::exception& e) {
                  recordCompileError("async", e.what());
                  return nullptr;
                }
              }).share();
  auto watched = std::async(std::launch::async, [this, work, key, timeout_ms]() -> std::shared_ptr<CompiledKernel> {
                   std::shared_ptr<CompiledKernel> k;
                   if (timeout_ms == 0 ||
                       work.wait_for(std::chrono::milliseconds(timeout_ms)) == std::future_status::ready) {
                     k = work.get();
                   } else {
                     recordCompileError("async-timeout", "compile exceeded " + std::to_string(timeout_ms) +
                                                             "ms for " + key);
                   }
                   std::lock_guard<std::mutex> l(state_->mu);
                   if (k) ++state_->async_completions;
                   else ++state_->async_failures;
                   state_->pending.erase(key);
                   return k;
                 }).share();
  state_->pending[key] = watched;
  state_->watchers.push_back(std::async(std::launch::deferred, [work]() { work.wait(); }));
  return watched;
}

std::vector<std::shared_ptr<CompiledKernel>> C3Engine::compileParallel(const std::vector<Graph>& graphs,
                                                                       const CompileOptions& options) {
  std::vector<std::future<std::shared_ptr<CompiledKernel>>> fs;
  for (const auto& g : graphs)
    fs.push_back(std::async(std::launch::async, [this, &g, &options]() { return compile(g, options); }));
  std::vector<std::shared_ptr<CompiledKernel>> out;
  for (auto& f : fs) out.push_back(f.get());
  return out;
}

std::shared_ptr<CompiledKernel> C3Engine::compileAndInject(const Graph& graph, const CompileOptions& options) {
  auto k = compile(graph, options);
  const Graph g = graph.eliminateDeadCode();
  const auto cn = g.computeNodes();
  if (cn.size() != 1) throw std::runtime_error("compileAndInject: single-op graphs only; pass op_type for regions");
  const auto& n = g.node(cn[0]);
  KernelShapeInfo info;
  info.out_shape = n.out_desc.shape;
  op o;
  if (std::holds_alternative<MatMulNode>(n.op)) {
    o = op::MatMul;
    info.is_matmul = true;
    info.lhs_shape = g.node(n.inputs[0]).out_desc.shape;
    info.rhs_shape = g.node(n.inputs[1]).out_desc.shape;
    info.M = info.out_shape[0];
    info.K = info.lhs_shape[1];
    info.N = info.out_shape[1];
  } else {
    static const std::unordered_map<std::string, op> byName = {
        {"Add", op::Add}, {"Sub", op::Sub}, {"Mul", op::Mul}, {"Div", op::Div}, {"Neg", op::Neg},
        {"ReLU", op::ReLU}, {"Sigmoid", op::Sigmoid}, {"Tanh", op::Tanh}, {"Exp", op::Exp}, {"Log", op::Log}};
    auto it = byName.find(nodeName(n.op));
    if (it == byName.end()) throw std::runtime_error("compileAndInject: cannot infer op type");
    o = it->second;
    info.lhs_shape = g.node(n.inputs[0]).out_desc.shape;
    if (n.inputs.size() > 1) info.rhs_shape = g.node(n.inputs[1]).out_desc.shape;
  }
  C3KernelRegistry::getInstance().install(o, DeviceType::kCUDA, k, info);
  C3KernelRegistry::getInstance().install(o, DeviceType::kCPU, k, info);
  return k;
}

std::shared_ptr<CompiledKernel> C3Engine::getKernel(const std::string& key) const {
  std::lock_guard<std::mutex> lock(state_->mu);
  auto it = state_->index.find(key);
  return it == state_->index.end() ? nullptr : it->second->second;
}

C3CacheStats C3Engine::getCacheStats() const {
  std::lock_guard<std::mutex> lock(state_->mu);
  C3CacheStats s;
  s.total_entries = state_->lru.size();
  s.hits = state_->hits;
  s.misses = state_->misses;
  s.evictions = state_->evictions;
  s.pending_compiles = state_->pending.size();
  s.async_completions = state_->async_completions;
  s.async_failures = state_->async_failures;
  for (const auto& [k, v] : state_->lru) s.bytes_used += k.size() + sizeof(*v);
  return s;
}

std::shared_ptr<ProfileData> C3Engine::getProfileData(const std::string& key) const {
  std::lock_guard<std::mutex> lock(state_->mu);
  auto it = state_->profiles.find(key);
  return it == state_->profiles.end() ? nullptr : it->second;
}

std::string C3Engine::getLastCompileError() const {
  std::lock_guard<std::mutex> lock(state_->mu);
  return state_->last_error;
}

void C3Engine::clearLastCompileError() {
  std::lock_guard<std::mutex> lock(state_->mu);
  state_->last_error.clear();
}

void C3Engine::recordCompileError(const std::string& prefix, const std::string& err) {
  std::string msg = prefix.empty() ? err : "[" + prefix + "] " + err;
  if (msg.size() > 1024) msg.resize(1024);
  {
    std::lock_guard<std::mutex> lock(state_->mu);
    state_->last_error = msg;
  }
  CtorchError::log(ErrorLevel::DEBUG, ErrorPlatform::kCUDA, ErrorType::RUNTIME, "C3Engine: " + msg);
}

bool C3Engine::wasAsyncCompileTimedOut(const std::string& cache_key) const {
  std::lock_guard<std::mutex> lock(state_->mu);
  const std::string& e = state_->last_error;
  return e.rfind("[async-timeout]", 0) == 0 &&
         e.find(cache_key.substr(0, std::min<size_t>(cache_key.size(), 900))) != std::string::npos;
}

void C3Engine::setCompileTimeoutMs(uint32_t ms) {
  std::lock_guard<std::mutex> lock(state_->mu);
  state_->timeout_ms = ms;
}

uint32_t C3Engine::getCompileTimeoutMs() const {
  std::lock_guard<std::mutex> lock(state_->mu);
  return state_->timeout_ms;
}

void C3Engine::clearCache() {
  std::lock_guard<std::mutex> lock(state_->mu);
  state_->lru.clear();
  state_->index.clear();
  state_->profiles.clear();
}

void C3Engine::shutdown() {
  std::vector<CompileFuture> pending;
  std::vector<std::future<void>> watchers;
  {
    std::lock_guard<std::mutex> lock(state_->mu);
    for (auto& [k, f] : state_->pending) pending.push_back(f);
    watchers.swap(state_->watchers);
  }
  for (auto& f : pending)
    if (f.valid() && f.wait_for(std::chrono::seconds(30)) != std::future_status::ready)
      CtorchError::log(ErrorLevel::WARN, ErrorPlatform::kGENERAL, ErrorType::UNKNOWN,
                       "C3Engine::shutdown: an async compile did not finish in 30 s");
  for (auto& w : watchers)
    if (w.valid()) w.get();
}

}  // namespace c3
}  // namespace ct
