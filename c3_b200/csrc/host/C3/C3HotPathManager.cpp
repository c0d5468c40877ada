#include "C3/C3HotPathManager.h"

#include <thread>

#include "C3/C3Config.h"
#include "C3/C3KernelRegistry.h"
#include "C3/RegionFusion.h"
#include "CtorchError.h"

namespace ct {
namespace c3 {

C3HotPathManager& C3HotPathManager::instance() {
  static C3HotPathManager mgr;
  return mgr;
}

C3HotPathManager::~C3HotPathManager() {
  shutting_down_.store(true, std::memory_order_release);
  std::vector<std::future<void>> fs;
  {
    std::lock_guard<std::mutex> lk(futures_mutex_);
    fs.swap(pending_futures_);
  }
  for (auto& f : fs)
    if (f.valid()) f.wait_for(std::chrono::milliseconds(100));
}

void C3HotPathManager::configure(const HotPathConfig& cfg) {
  std::lock_guard<std::mutex> lk(cfg_mutex_);
  config_ = cfg;
}

HotPathConfig C3HotPathManager::getConfig() const {
  std::lock_guard<std::mutex> lk(cfg_mutex_);
  return config_;
}

C3HotPathManager::Stats C3HotPathManager::getStats() const {
  Stats s;
  s.calls_tracked = calls_tracked_.load(std::memory_order_relaxed);
  s.compilations_triggered = compilations_triggered_.load(std::memory_order_relaxed);
  s.pending_compiles = pending_compiles_.load(std::memory_order_relaxed);
  std::lock_guard<std::mutex> lk(mutex_);
  s.cooldown_hits = cooldown_hits_;
  s.backpressure_hits = backpressure_hits_;
  return s;
}

void C3HotPathManager::track(std::future<void> f) {
  std::lock_guard<std::mutex> lk(futures_mutex_);
  pending_futures_.push_back(std::move(f));
}

void C3HotPathManager::shutdown() {
  shutting_down_.store(true, std::memory_order_release);
  std::vector<std::future<void>> fs;
  {
    std::lock_guard<std::mutex> lk(futures_mutex_);
    fs.swap(pending_futures_);
  }
  for (auto& f : fs) {
    if (!f.valid()) continue;
    if (f.wait_for(std::chrono::seconds(30)) == std::future_status::ready) {
      try {
        f.get();
      } catch (...) {
      }
    } else {
      CtorchError::log(ErrorLevel::WARN, ErrorPlatform::kGENERAL, ErrorType::UNKNOWN,
                       "C3HotPathManager::shutdown: background compile did not finish in 30s");
    }
  }
}

void C3HotPathManager::waitForPendingCompiles() {
  while (pending_compiles_.load(std::memory_order_acquire) > 0)
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  std::vector<std::future<void>> fs;
  {
    std::lock_guard<std::mutex> lk(futures_mutex_);
    fs.swap(pending_futures_);
  }
  for (auto& f : fs)
    if (f.valid()) f.wait();
}

void C3HotPathManager::clear() {
  std::lock_guard<std::mutex> lk(mutex_);
  entries_.clear();
  std::lock_guard<std::mutex> rb(rb_mutex_);
  recent_dispatches_.clear();
  calls_tracked_.store(0);
  compilations_triggered_.store(0);
  pending_compiles_.store(0);
  cooldown_hits_ = 0;
  backpressure_hits_ = 0;
  shutting_down_.store(false, std::memory_order_release);
}

size_t C3HotPathManager::hashShapeKey(const std::vector<size_t>& shape, op op_type, DeviceType dev) {
  size_t h = static_cast<size_t>(op_type) ^ (static_cast<size_t>(dev) << 8);
  h ^= 0x9e3779b9 + (h << 6) + (h >> 2);
  for (auto s : shape) h ^= s + 0x9e3779b9 + (h << 6) + (h >> 2);
  return h;
}

bool C3HotPathManager::isSupportedOp(op o) {
  static constexpr uint64_t kMask =
      (1ull << static_cast<size_t>(op::Add)) | (1ull << static_cast<size_t>(op::Sub)) |
      (1ull << static_cast<size_t>(op::Mul)) | (1ull << static_cast<size_t>(op::Div)) |
      (1ull << static_cast<size_t>(op::MatMul)) | (1ull << static_cast<size_t>(op::Neg)) |
      (1ull << static_cast<size_t>(op::ReLU)) | (1ull << static_cast<size_t>(op::Tanh)) |
      (1ull << static_cast<size_t>(op::Sigmoid));
  return (kMask >> static_cast<size_t>(o)) & 1ull;
}

bool C3HotPathManager::isUnaryOp(op o) {
  switch (o) {
    case op::Neg: case op::ReLU: case op::Tanh: case op::Sigmoid: case op::GELU: case op::LReLU:
    case op::Log: case op::Exp: case op::Abs: case op::Sin: case op::Cos:
      return true;
    default:
      return false;
  }
}

std::vector<size_t> C3HotPathManager::extractBinOpOutShape(const std::vector<size_t>& shape) {
  if (shape.size() >= 4) return {shape[0], shape[shape.size() - 1]};
  if (shape.size() >= 2) return {shape[0], shape[1]};
  return shape;
}

void C3HotPathManager::recordCall(op op_type, DeviceType dev, const std::vector<size_t>& lhs_shape,
                                  const std::vector<size_t>& rhs_shape, bool in_autograd) {
  if (!hotPathTrackingEnabled()) return;
  calls_tracked_.fetch_add(1, std::memory_order_relaxed);
  if (dev == DeviceType::kMPS) return;
  if (shutting_down_.load(std::memory_order_acquire)) return;

  std::vector<size_t> shape = lhs_shape;
  shape.insert(shape.end(), rhs_shape.begin(), rhs_shape.end());
  {
    std::lock_guard<std::mutex> lk(rb_mutex_);
    recent_dispatches_.push_back({op_type, shape, lhs_shape, rhs_shape, std::chrono::steady_clock::now()});
    if (recent_dispatches_.size() > kMaxRingBufferSize) recent_dispatches_.pop_front();
  }
  const HotPathConfig cfg = getConfig();
  if (in_autograd) {
    // training: region detection only, no single-op compiles
    tryFuseRecentDispatches(dev, cfg);
    return;
  }
  const size_t key = hashShapeKey(shape, op_type, dev);
  bool should_compile = false;
  {
    std::lock_guard<std::mutex> lk(mutex_);
    auto& e = entries_[key];
    e.call_count++;
    const auto elapsed = std::chrono::duration_cast<std::chrono::seconds>(
                             std::chrono::steady_clock::now() - e.last_compile_time)
                             .count();
    if (e.last_compile_time.time_since_epoch().count() != 0 &&
        elapsed < static_cast<decltype(elapsed)>(cfg.cooldown_sec)) {
      cooldown_hits_++;
      return;
    }
    if (pending_compiles_.load(std::memory_order_relaxed) >= cfg.max_pending) {
      backpressure_hits_++;
      return;
    }
    if (e.call_count >= cfg.hot_threshold && !e.compiling) {
      e.compiling = true;
      e.call_count = 0;
      pending_compiles_.fetch_add(1, std::memory_order_relaxed);
      compilations_triggered_.fetch_add(1, std::memory_order_relaxed);
      should_compile = true;
    }
  }
  if (should_compile) {
    tryFuseRecentDispatches(dev, cfg);
    submitCompileAsync(op_type, dev, shape, lhs_shape, rhs_shape, key, cfg);
  }
}

void C3HotPathManager::tryFuseRecentDispatches(DeviceType dev, const HotPathConfig& cfg) {
  std::vector<DispatchRecord> recs;
  std::string pattern;
  {
    std::lock_guard<std::mutex> lk(rb_mutex_);
    const auto& q = recent_dispatches_;
    if (q.size() < 2) return;
    auto matmul_ok = [](const DispatchRecord& r) { return r.op_type == op::MatMul && r.shape.size() >= 4; };
    if (q.size() >= 3) {
      const auto& a = q[q.size() - 3];
      const auto& b = q[q.size() - 2];
      const auto& c = q[q.size() - 1];
      if (matmul_ok(a) && b.op_type == op::Add && b.shape.size() >= 2 &&
          (c.op_type == op::ReLU || c.op_type == op::Sigmoid) && !c.shape.empty() &&
          b.shape[0] == a.shape[0] && b.shape[1] == a.shape[3]) {
        recs = {a, b, c};
        pattern = c.op_type == op::ReLU ? "MatMul+Add+ReLU" : "MatMul+Add+Sigmoid";
      }
    }
    if (recs.empty()) {
      const auto& a = q[q.size() - 2];
      const auto& c = q[q.size() - 1];
      if (matmul_ok(a) && (c.op_type == op::ReLU || c.op_type == op::Sigmoid) && !c.shape.empty()) {
        const size_t M = a.shape[0], N = a.shape[3];
        const bool ok = c.shape.size() >= 2 ? (c.shape[0] == M && c.shape[1] == N) : (c.shape[0] == M * N);
        if (ok) {
          recs = {a, c};
          pattern = c.op_type == op::ReLU ? "MatMul+ReLU" : "MatMul+Sigmoid";
        }
      }
    }
  }
  if (!recs.empty()) submitFusedCompileAsync(recs, dev, cfg, pattern);
}

Graph C3HotPathManager::buildGraphForOp(op o, const std::vector<size_t>& shape, const std::vector<size_t>& lhs,
                                        const std::vector<size_t>& rhs) {
  Graph g;
  auto unary = [&](NodeVariant v) {
    auto d = TensorDesc::fromShape(lhs);
    const size_t in = g.addInput(d);
    g.markOutput(g.addNode(std::move(v), {in}, d));
  };
  auto binary = [&](auto node_t) {
    auto l = TensorDesc::fromShape(lhs);
    auto r = TensorDesc::fromShape(rhs.empty() ? lhs : rhs);
    const size_t a = g.addInput(l), b = g.addInput(r);
    node_t.lhs_desc = l;
    node_t.rhs_desc = r;
    g.markOutput(g.addNode(node_t, {a, b}, l));
  };
  switch (o) {
    case op::Sigmoid: unary(SigmoidNode{TensorDesc::fromShape(lhs)}); break;
    case op::Tanh: unary(TanhNode{TensorDesc::fromShape(lhs)}); break;
    case op::ReLU: unary(ReLUNode{TensorDesc::fromShape(lhs)}); break;
    case op::Neg: unary(NegNode{TensorDesc::fromShape(lhs)}); break;
    case op::Add: binary(AddNode{}); break;
    case op::Sub: binary(SubNode{}); break;
    case op::Mul: binary(MulNode{}); break;
    case op::Div: binary(DivNode{}); break;
    case op::MatMul:
      if (shape.size() >= 4 && shape[1] == shape[2]) {
        auto l = TensorDesc::fromShape({shape[0], shape[1]});
        auto r = TensorDesc::fromShape({shape[2], shape[3]});
        const size_t a = g.addInput(l), b = g.addInput(r);
        g.markOutput(g.addNode(MatMulNode{l, r}, {a, b}, TensorDesc::fromShape({shape[0], shape[3]})));
      }
      break;
    default:
      break;
  }
  return g;
}

Graph C3HotPathManager::buildFusedGraph(const std::vector<DispatchRecord>& records, const std::string&) {
  // MatMul(X[M,K], B[K,N]) -> [Add(., bias)] -> act; external inputs in record order:
  // X, B, then the Add's rhs (the region kernel's {X, B, b}).
  Graph g;
  if (records.empty() || records[0].op_type != op::MatMul || records[0].shape.size() < 4) return g;
  const auto& r0 = records[0];
  const size_t M = r0.shape[0], K = r0.shape[1], N = r0.shape[3];
  auto lhs = TensorDesc::fromShape({M, K}), rhs = TensorDesc::fromShape({K, N});
  auto out = TensorDesc::fromShape({M, N});
  const size_t x = g.addInput(lhs), b = g.addInput(rhs);
  std::vector<std::pair<size_t, std::vector<size_t>>> extra;  // record index -> rhs shape
  for (size_t i = 1; i < records.size(); ++i)
    if (!isUnaryOp(records[i].op_type)) {
      const auto os = extractBinOpOutShape(records[i].shape);
      std::vector<size_t> rs = records[i].shape.size() > os.size()
                                   ? std::vector<size_t>(records[i].shape.begin() + static_cast<long>(os.size()),
                                                         records[i].shape.end())
                                   : os;
      extra.push_back({i, rs});
    }
  std::unordered_map<size_t, size_t> ext_input;
  for (const auto& [i, rs] : extra) ext_input[i] = g.addInput(TensorDesc::fromShape(rs));
  size_t prev = g.addNode(MatMulNode{lhs, rhs}, {x, b}, out);
  for (size_t i = 1; i < records.size(); ++i) {
    const op o = records[i].op_type;
    if (o == op::Add) {
      const size_t in = ext_input[i];
      prev = g.addNode(AddNode{out, g.node(in).out_desc}, {prev, in}, out);
    } else if (o == op::ReLU) {
      prev = g.addNode(ReLUNode{out}, {prev}, out);
    } else if (o == op::Sigmoid) {
      prev = g.addNode(SigmoidNode{out}, {prev}, out);
    } else if (o == op::Tanh) {
      prev = g.addNode(TanhNode{out}, {prev}, out);
    } else {
      return Graph();  // not a region pattern
    }
  }
  g.markOutput(prev);
  return g;
}

void C3HotPathManager::submitFusedCompileAsync(const std::vector<DispatchRecord>& records, DeviceType dev,
                                               const HotPathConfig& cfg, const std::string& pattern) {
  size_t fused_key = 0;
  for (const auto& r : records) fused_key ^= hashShapeKey(r.shape, r.op_type, dev);
  {
    std::lock_guard<std::mutex> lk(mutex_);
    auto it = entries_.find(fused_key);
    if (it != entries_.end() && it->second.compiling) return;
    if (it != entries_.end() && it->second.last_compile_time.time_since_epoch().count() != 0 &&
        std::chrono::duration_cast<std::chrono::seconds>(std::chrono::steady_clock::now() -
                                                         it->second.last_compile_time)
                .count() < static_cast<long>(cfg.cooldown_sec))
      return;
    entries_[fused_key].compiling = true;
  }
  pending_compiles_.fetch_add(1, std::memory_order_relaxed);
  compilations_triggered_.fetch_add(1, std::memory_order_relaxed);
  if (cfg.verbose)
    CtorchError::log(ErrorLevel::INFO, ErrorPlatform::kGENERAL, ErrorType::UNKNOWN,
                     "C3HotPathManager: fusion pattern detected: " + pattern);
  track(std::async(std::launch::async, [this, records, fused_key, pattern, dev]() {
    try {
      Graph g = buildFusedGraph(records, pattern);
      CompileOptions opts;
      auto kernel = g.outputCount() ? C3Engine::getInstance().compile(g, opts) : nullptr;
      if (kernel) {
        KernelShapeInfo info;
        const auto& r0 = records[0];
        info.lhs_shape = {r0.shape[0], r0.shape[1]};
        info.rhs_shape = {r0.shape[2], r0.shape[3]};
        info.out_shape = extractBinOpOutShape(records.back().shape);
        info.is_matmul = true;
        info.M = r0.shape[0];
        info.K = r0.shape[1];
        info.N = r0.shape[3];
        info.fused_pattern = pattern;
        C3KernelRegistry::getInstance().installFused(kernel, records.back().op_type, info);
        std::vector<op> seq;
        std::vector<size_t> numels;
        for (const auto& r : records) {
          seq.push_back(r.op_type);
          size_t n = 1;
          for (auto s : extractBinOpOutShape(r.shape)) n *= s;
          numels.push_back(n);
        }
        RegionFusionRegistry::getInstance().installWithCost(seq, kernel, numels,
                                                            {{r0.shape[0], r0.shape[1]}, {r0.shape[2], r0.shape[3]}});
      }
    } catch (const std::exception& e) {
      C3Engine::getInstance().recordCompileError("fused", e.what());
    }
    (void)dev;
    pending_compiles_.fetch_sub(1, std::memory_order_relaxed);
    std::lock_guard<std::mutex> lk(mutex_);
    auto it = entries_.find(fused_key);
    if (it != entries_.end()) {
      it->second.compiling = false;
      it->second.last_compile_time = std::chrono::steady_clock::now();
    }
  }));
}

void C3HotPathManager::submitCompileAsync(op op_type, DeviceType dev, const std::vector<size_t>& shape,
                                          const std::vector<size_t>& lhs, const std::vector<size_t>& rhs,
                                          size_t key, const HotPathConfig& cfg) {
  auto release = [this, key]() {
    pending_compiles_.fetch_sub(1, std::memory_order_relaxed);
    std::lock_guard<std::mutex> lk(mutex_);
    auto it = entries_.find(key);
    if (it != entries_.end()) {
      it->second.compiling = false;
      it->second.last_compile_time = std::chrono::steady_clock::now();
    }
  };
  if (!isSupportedOp(op_type) || !singleKernelInjectionEnabled()) {
    release();
    return;
  }
  Graph g = buildGraphForOp(op_type, shape, lhs, rhs);
  if (g.outputCount() == 0) {
    release();
    return;
  }
  auto& engine = C3Engine::getInstance();
  engine.setCompileTimeoutMs(cfg.compile_timeout_ms);
  // Two tiers as in the reference (opt 2, then opt 4); both bind the same B200 kernel, and
  // the registry keeps the higher level.
  CompileOptions fast;
  fast.opt_level = 2;
  CompileOptions extreme;
  extreme.opt_level = 4;
  auto f_fast = engine.compileAsync(g, fast);
  auto f_ext = engine.compileAsync(g, extreme);
  auto install = [op_type, shape, lhs, rhs, dev](const std::shared_ptr<CompiledKernel>& k) {
    if (!k) return;
    KernelShapeInfo info;
    if (op_type == op::MatMul && shape.size() >= 4) {
      info.is_matmul = true;
      info.M = shape[0];
      info.K = shape[1];
      info.N = shape[3];
      info.lhs_shape = {shape[0], shape[1]};
      info.rhs_shape = {shape[1], shape[3]};
      info.out_shape = {shape[0], shape[3]};
    } else {
      info.lhs_shape = lhs;
      info.rhs_shape = rhs;
      info.out_shape = lhs;
    }
    C3KernelRegistry::getInstance().install(op_type, dev, k, info);
  };
  track(std::async(std::launch::async, [f_fast, f_ext, install, release]() {
    install(f_fast.get());
    install(f_ext.get());
    release();
  }));
}

}  // namespace c3
}  // namespace ct
