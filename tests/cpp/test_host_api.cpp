// Tests of the C++ mirror of the C3 install-and-dispatch API (c3_b200/csrc/host).
//
//   test_host_api --cpu   host logic only: rolling hash and region keys (known answers derived
//                         from the reference code), cost model, registry install / preemption /
//                         fallback semantics, graph lowering, hot-path trigger, backward keys
//   test_host_api --gpu   the same API driving the sm_100a kernels, checked against the oracle
//                         (liboracle.so, test infrastructure)
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <array>
#include <atomic>
#include <chrono>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "AutoGrad/Node.h"
#include "C3/C3BackwardCapture.h"
#include "C3/C3Cleanup.h"
#include "C3/C3Engine.h"
#include "C3/C3HotPathManager.h"
#include "C3/C3KernelRegistry.h"
#include "C3/CudaKernels.h"
#include "C3/CudaRuntime.h"
#include "C3/FusionCostModel.h"
#include "C3/RegionFusion.h"
#include "C3/RollingHash.h"
#include "c3cu.h"
#include "gemm2_schedule.h"

extern "C" {
void c3o_region_fwd(const float* X, const float* B, const float* b, size_t b_numel, float* out, float* z,
                    size_t M, size_t K, size_t N, int transB, size_t r0, size_t r1, int threads);
void c3o_matmul(const float* A, const float* B, float* out, size_t M, size_t K, size_t N, int transA,
                int transB, const float* bias, size_t bias_numel, int act, size_t r0, size_t r1, int threads);
void c3o_relu_bwd(const float* grad, const float* x, float* out, size_t n);
void c3o_sum_reduce(const float* in, float* out, size_t M, size_t N, int axis);
void c3o_backward_chain(const int* ops, int n_nodes, const float* grad, const float* const* xs, float* const* outs,
                        size_t n);
}

// Graph node structs and the host framework's autograd node classes share names
// (ReLUNode, AddNode, MatMulNode, ...): graph nodes are spelled c3::X, autograd nodes ::X.
namespace c3 = ct::c3;
using c3::C3BackwardCapture;
using c3::C3Engine;
using c3::C3HotPathManager;
using c3::C3KernelRegistry;
using c3::CompiledKernel;
using c3::CudaKernelBase;
using c3::FusionCostModel;
using c3::Graph;
using c3::HotPathConfig;
using c3::KernelShapeInfo;
using c3::RegionEntry;
using c3::RegionFusionRegistry;
using c3::RollingHash;
using c3::TensorDesc;
using c3::shutdownAll;

static int g_failures = 0, g_checks = 0;
#define CHECK(cond)                                                               \
  do {                                                                            \
    ++g_checks;                                                                   \
    if (!(cond)) {                                                                \
      ++g_failures;                                                               \
      std::fprintf(stderr, "  CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond); \
    }                                                                             \
  } while (0)

struct TestCase {
  const char* name;
  bool gpu;
  std::function<void()> fn;
};
static std::vector<TestCase>& registry() {
  static std::vector<TestCase> r;
  return r;
}
struct Reg {
  Reg(const char* n, bool gpu, std::function<void()> f) { registry().push_back({n, gpu, std::move(f)}); }
};
#define TEST(name, gpu) \
  static void name();   \
  static Reg reg_##name(#name, gpu, name); \
  static void name()

// A CPU-only CompiledKernel used to exercise the registries without a device.
class FakeKernel : public CompiledKernel {
 public:
  FakeKernel(int level, std::vector<size_t> out, bool fail = false) : out_(std::move(out)), fail_(fail) {
    opt_level_ = level;
  }
  std::vector<Tensor> execute(const std::vector<Tensor>&) override {
    ++calls;
    if (fail_) throw std::runtime_error("fake failure");
    Tensor t(ShapeTag{}, out_, DType::kFloat, DeviceType::kCPU);
    for (size_t i = 0; i < t.numel(); ++i) t.data_write<float>()[i] = static_cast<float>(opt_level_);
    return {t};
  }
  const std::string& cacheKey() const override { return key_; }
  DeviceType targetDevice() const override { return DeviceType::kCPU; }
  size_t workspaceBytes() const override { return 0; }
  int calls = 0;

 private:
  std::vector<size_t> out_;
  bool fail_;
  std::string key_ = "fake";
};

static Tensor hostTensor(const std::vector<size_t>& shape, std::mt19937& rng, float lo, float hi) {
  Tensor t(ShapeTag{}, shape, DType::kFloat, DeviceType::kCPU);
  std::uniform_real_distribution<float> d(lo, hi);
  for (size_t i = 0; i < t.numel(); ++i) t.data_write<float>()[i] = d(rng);
  return t;
}

static Graph regionGraph(size_t M, size_t K, size_t N) {
  Graph g;
  auto x = TensorDesc::fromShape({M, K}), b = TensorDesc::fromShape({K, N}), o = TensorDesc::fromShape({M, N});
  auto bias = TensorDesc::fromShape({N});
  const size_t xi = g.addInput(x), bi = g.addInput(b), ci = g.addInput(bias);
  const size_t mm = g.addNode(c3::MatMulNode{x, b}, {xi, bi}, o);
  const size_t add = g.addNode(c3::AddNode{o, bias}, {mm, ci}, o);
  g.markOutput(g.addNode(c3::ReLUNode{o}, {add}, o));
  return g;
}

// ============================================================================ CPU
// The CTA-pair GEMM's work schedule (the launcher's split plan and the kernel's per-cluster
// items, c3_b200/csrc/gemm2_schedule.h) over every cluster count a B200 launch can have
// (1..74, including SM caps) and a sweep of tile counts and K depths: every output tile's K
// range is computed exactly once, either whole or as two non-empty halves on the two clusters
// that share its split slot; no launched cluster is idle; the slot fits the workspace.
TEST(gemm2_schedule_covers_every_tile_once, false) {
  using c3cu::gemm2::Item;
  const int split_slots = 80;
  std::vector<int> tile_counts;
  for (int t = 1; t <= 400; ++t) tile_counts.push_back(t);
  for (int t : {512, 1024, 1152, 4096}) tile_counts.push_back(t);
  std::vector<std::array<Item, 3>> seen;
  std::vector<int> nseen;
  long configs = 0, bad = 0;
  for (int variant : {0, 2})
    for (int kb : {1, 2, 63, 64, 65, 127, 128})
      for (int maxc = 1; maxc <= 74; ++maxc)
        for (int tiles : tile_counts) {
          ++configs;
          const auto plan = c3cu::gemm2::plan_split(tiles, maxc, kb, variant, split_slots);
          bool ok = plan.clusters >= 1 && plan.clusters <= maxc && (plan.sk_mode == 0 || plan.sk_mode == 1);
          if (plan.sk_mode == 1) ok = ok && variant == 0 && kb >= 64 && plan.sk_first >= 0 && plan.sk_first < tiles;
          seen.assign(tiles, {});
          nseen.assign(tiles, 0);
          for (int c = 0; ok && c < plan.clusters; ++c) {
            Item it{};
            int i = 0;
            for (; c3cu::gemm2::work_item(i, c, plan.clusters, tiles, plan.sk_mode, plan.sk_first, kb, it); ++i) {
              if (it.tile < 0 || it.tile >= tiles || nseen[it.tile] >= 2) { ok = false; break; }
              Item rec = it;
              rec.split = it.split < 0 ? -1 : (it.split << 8) | c;  // remember the cluster too
              seen[it.tile][nseen[it.tile]++] = rec;
            }
            if (i == 0) ok = false;  // a launched cluster with no work
          }
          for (int t = 0; ok && t < tiles; ++t) {
            if (nseen[t] == 1) {
              const Item& a = seen[t][0];
              ok = a.kb0 == 0 && a.kb1 == kb && a.split == -1;
            } else if (nseen[t] == 2) {
              Item a = seen[t][0], b = seen[t][1];
              if (a.kb0 > b.kb0) std::swap(a, b);
              const int slot = a.split >> 8;
              ok = plan.sk_mode == 1 && a.split >= 0 && b.split >= 0 && slot == (b.split >> 8) &&
                   slot == t - plan.sk_first && slot < split_slots && a.kb0 == 0 && a.kb1 == b.kb0 &&
                   b.kb1 == kb && a.kb1 > 0 && b.kb0 < kb && (a.split & 0xff) == 2 * slot &&
                   (b.split & 0xff) == 2 * slot + 1;
            } else {
              ok = false;
            }
          }
          if (!ok && ++bad <= 5)
            std::fprintf(stderr, "  schedule wrong: variant %d, k_blocks %d, clusters %d, tiles %d\n", variant,
                         kb, maxc, tiles);
        }
  CHECK(bad == 0);
  CHECK(configs > 400000);
  // the cfg3 dW GEMM: 256 tiles on 74 pairs splits the 34 tail tiles over 68 clusters
  const auto dw = c3cu::gemm2::plan_split(256, 74, 64, 0, split_slots);
  CHECK(dw.sk_mode == 1 && dw.sk_first == 222 && dw.clusters == 74);
  // K = 2048 (32 blocks) never splits
  CHECK(c3cu::gemm2::plan_split(256, 74, 32, 0, split_slots).sk_mode == 0);
}

// Kernel for the concurrency stress test: an atomic call count, output filled with its level.
class CountingKernel : public CompiledKernel {
 public:
  CountingKernel(int level, std::vector<size_t> out) : out_(std::move(out)) { opt_level_ = level; }
  std::vector<Tensor> execute(const std::vector<Tensor>&) override {
    calls.fetch_add(1, std::memory_order_relaxed);
    Tensor t(ShapeTag{}, out_, DType::kFloat, DeviceType::kCPU);
    for (size_t i = 0; i < t.numel(); ++i) t.data_write<float>()[i] = static_cast<float>(opt_level_);
    return {t};
  }
  const std::string& cacheKey() const override { return key_; }
  DeviceType targetDevice() const override { return DeviceType::kCPU; }
  size_t workspaceBytes() const override { return 0; }
  std::atomic<int> calls{0};

 private:
  std::vector<size_t> out_;
  std::string key_ = "counting";
};

// Dispatch threads look kernels up and run them while a compile thread installs ever higher
// tiers into the single-op registry and reinstalls the same region key, as the reference's
// background compiles do (a tuned tier replacing the precompiled one). Checks: no dispatcher
// ever sees an uninstalled op or a half-written entry, tiers only move up for each dispatcher,
// hit counters add up, and the last install wins. Under ThreadSanitizer (tests run the binary
// built with -fsanitize=thread on this test) it also shows the registries free of data races.
TEST(registries_concurrent_install_and_dispatch, false) {
  auto& reg = C3KernelRegistry::getInstance();
  auto& rr = RegionFusionRegistry::getInstance();
  reg.uninstallAll();
  rr.clear();
  const KernelShapeInfo info{{4, 4}, {4, 4}, {4, 4}};
  const std::vector<op> seq{op::MatMul, op::Add, op::ReLU};
  const std::vector<std::vector<size_t>> shapes{{4, 4}, {4, 4}};
  const uint64_t rkey = RegionFusionRegistry::regionKey(seq, shapes);
  std::mt19937 rng(3);
  const Tensor a = hostTensor({4, 4}, rng, -1, 1), b = hostTensor({4, 4}, rng, -1, 1);
  constexpr int kReaders = 6, kIters = 2000, kLevels = 8;
  std::vector<std::shared_ptr<CountingKernel>> kernels;
  for (int l = 1; l <= kLevels; ++l) kernels.push_back(std::make_shared<CountingKernel>(l, std::vector<size_t>{4, 4}));
  std::atomic<bool> go{false};
  std::atomic<long> hits{0}, region_runs{0}, bad{0};
  const size_t hits_before = reg.getStats().hit_count;
  std::vector<std::thread> threads;
  for (int r = 0; r < kReaders; ++r)
    threads.emplace_back([&] {
      while (!go.load()) std::this_thread::yield();
      int last = 0;
      for (int i = 0; i < kIters; ++i) {
        if (auto out = reg.tryExecute(op::Add, a, b)) {
          const int v = static_cast<int>(out->data_read<float>()[0]);
          hits.fetch_add(1);
          if (v < last || v < 1 || v > kLevels) bad.fetch_add(1);
          last = v;
        }
        if (reg.tryExecute(op::Div, a, b)) bad.fetch_add(1);  // never installed
        if (rr.mayMatchAsLastOp(op::ReLU)) {
          if (RegionEntry* e = rr.find(rkey)) {
            std::shared_ptr<CompiledKernel> k = e->kernel;  // the read a host dispatcher makes
            if (!k || e->op_seq != seq || !e->active)
              bad.fetch_add(1);
            else if (k->execute({a, b}).size() == 1)
              region_runs.fetch_add(1);
          }
        }
      }
    });
  threads.emplace_back([&] {
    while (!go.load()) std::this_thread::yield();
    for (int l = 0; l < kLevels; ++l) {
      reg.install(op::Add, DeviceType::kCPU, kernels[l], info);   // preempts the previous tier
      reg.install(op::Add, DeviceType::kCPU, kernels[0], info);   // lower tier: ignored
      rr.installWithCost(seq, kernels[l], {16, 16, 16}, shapes);  // reinstall under the same key
      std::this_thread::sleep_for(std::chrono::microseconds(300));
    }
  });
  go.store(true);
  for (auto& t : threads) t.join();
  CHECK(bad.load() == 0);
  CHECK(hits.load() > 0 && region_runs.load() > 0);
  CHECK(reg.getStats().hit_count - hits_before == static_cast<size_t>(hits.load()));
  auto final_out = reg.tryExecute(op::Add, a, b);
  CHECK(final_out && final_out->data_read<float>()[0] == static_cast<float>(kLevels));
  RegionEntry* e = rr.find(rkey);
  CHECK(e != nullptr && e->kernel == kernels.back());
  reg.uninstallAll();
  rr.clear();
}

// Several dispatch threads record MatMul -> Add -> ReLU sequences of their own shapes into the
// hot-path manager (one ring buffer for all threads) while its background compiles install the
// detected regions, and query both registries as they go. Checks: every region a dispatcher
// finds is complete, compiles were triggered and all finish, and the counters add up. Run under
// ThreadSanitizer too (with the registries' test) for the manager's own locking.
TEST(hot_path_concurrent_record_and_compile, false) {
  auto& hp = C3HotPathManager::instance();
  hp.clear();
  HotPathConfig cfg;
  cfg.hot_threshold = 2;
  hp.configure(cfg);
  auto& rr = RegionFusionRegistry::getInstance();
  auto& reg = C3KernelRegistry::getInstance();
  rr.clear();
  reg.uninstallAll();
  constexpr int kThreads = 4, kRounds = 150;
  std::atomic<bool> go{false};
  std::atomic<long> found{0}, bad{0};
  const size_t tracked_before = hp.getStats().calls_tracked;
  std::vector<std::thread> threads;
  for (int t = 0; t < kThreads; ++t)
    threads.emplace_back([&, t] {
      while (!go.load()) std::this_thread::yield();
      const size_t M = 64 * static_cast<size_t>(t + 1);
      const uint64_t key = RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{M, 784}, {784, 256}});
      for (int i = 0; i < kRounds; ++i) {
        hp.recordCall(op::MatMul, DeviceType::kCUDA, {M, 784}, {784, 256}, true);
        hp.recordCall(op::Add, DeviceType::kCUDA, {M, 256}, {256}, true);
        hp.recordCall(op::ReLU, DeviceType::kCUDA, {M, 256}, {}, true);
        if (rr.mayMatchAsLastOp(op::ReLU)) {
          if (RegionEntry* e = rr.find(key)) {
            std::shared_ptr<CompiledKernel> k = e->kernel;
            if (e->len != 3 || !k || !e->cost.worthwhile) bad.fetch_add(1); else found.fetch_add(1);
          }
        }
        (void)reg.findFusedKernelForSequence({op::MatMul, op::Add, op::ReLU}, DeviceType::kCUDA, {M, 784});
        (void)hp.getStats();
      }
    });
  go.store(true);
  for (auto& th : threads) th.join();
  hp.waitForPendingCompiles();
  const auto st = hp.getStats();
  CHECK(bad.load() == 0);
  CHECK(st.calls_tracked - tracked_before == static_cast<size_t>(kThreads) * kRounds * 3);
  CHECK(st.pending_compiles == 0);
  // at least one thread's own shapes end up installed (its sequence is found uninterleaved)
  size_t installed = 0;
  for (int t = 0; t < kThreads; ++t) {
    const size_t M = 64 * static_cast<size_t>(t + 1);
    installed += rr.find(RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{M, 784}, {784, 256}})) != nullptr;
  }
  CHECK(installed >= 1);
  hp.shutdown();
  hp.clear();
  rr.clear();
  reg.uninstallAll();
}

TEST(rolling_hash_known_answers, false) {
  // ((13*131)+2)*131+29 for {MatMul, Add, ReLU} (codes MatMul 13, Add 2, ReLU 29)
  CHECK(RollingHash::hashSequence({op::MatMul, op::Add, op::ReLU}) == 223384ull);
  CHECK(RollingHash::getOpCode(op::Sigmoid) == 37 && RollingHash::getOpCode(op::kCount) == 101);
  auto p = RollingHash::computePrefixHashes({op::Add, op::MatMul, op::Add, op::ReLU});
  CHECK(RollingHash::getSubHash(p, 1, 3) == 223384ull);
  CHECK(RollingHash::getSubHash(p, 0, 0) == 2ull);
}

TEST(region_key_mixes_first_input_shape, false) {
  // shape_hash over {128, 784}: (0*31 + 128 + 1)*31 + 784 + 1 = 4784
  const uint64_t k = RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{128, 784}, {784, 256}});
  CHECK(k == (223384ull ^ (4784ull << 32)));
  CHECK(RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {}) == 223384ull);
}

TEST(cost_model_known_answers, false) {
  auto c = FusionCostModel::estimate({op::MatMul, op::Add, op::ReLU}, {100, 100, 100});
  CHECK(c.eager_accesses == 500 && c.saved_accesses == 200 && c.fused_accesses == 300);
  CHECK(std::fabs(c.gain_ratio - 0.4) < 1e-12 && c.worthwhile);
  auto m = FusionCostModel::estimate({op::MatMul, op::ReLU}, {100, 100});
  CHECK(m.saved_accesses == 0 && !m.worthwhile);  // MatMul intermediate saves nothing
  CHECK(!FusionCostModel::estimate({}, {}).worthwhile);
}

TEST(registry_preemption_and_fallback, false) {
  auto& reg = C3KernelRegistry::getInstance();
  reg.uninstallAll();
  KernelShapeInfo info{{4, 4}, {4, 4}, {4, 4}};
  auto lo = std::make_shared<FakeKernel>(2, std::vector<size_t>{4, 4});
  auto hi = std::make_shared<FakeKernel>(4, std::vector<size_t>{4, 4});
  reg.install(op::Add, DeviceType::kCPU, hi, info);
  reg.install(op::Add, DeviceType::kCPU, lo, info);  // lower level: ignored
  std::mt19937 rng(1);
  Tensor a = hostTensor({4, 4}, rng, -1, 1), b = hostTensor({4, 4}, rng, -1, 1);
  auto r = reg.tryExecute(op::Add, a, b);
  CHECK(r.has_value() && r->data_read<float>()[0] == 4.0f && lo->calls == 0);
  // shape mismatch -> nullopt without executing
  Tensor c = hostTensor({4, 5}, rng, -1, 1);
  CHECK(!reg.tryExecute(op::Add, a, c).has_value());
  // a throwing kernel -> nullopt, counted as a miss
  auto bad = std::make_shared<FakeKernel>(5, std::vector<size_t>{4, 4}, true);
  reg.install(op::Mul, DeviceType::kCPU, bad, info);
  const auto before = reg.getStats().miss_count;
  CHECK(!reg.tryExecute(op::Mul, a, b).has_value());
  CHECK(reg.getStats().miss_count == before + 1);
  // wrong output shape uninstalls the kernel
  auto wrong = std::make_shared<FakeKernel>(5, std::vector<size_t>{2, 2});
  reg.install(op::Sub, DeviceType::kCPU, wrong, info);
  CHECK(!reg.tryExecute(op::Sub, a, b).has_value());
  CHECK(!reg.tryExecute(op::Sub, a, b).has_value() && wrong->calls == 1);
  reg.uninstallAll();
  CHECK(reg.getStats().active_entries == 0);
}

TEST(backward_entries_use_fwd_input_map, false) {
  auto& reg = C3KernelRegistry::getInstance();
  reg.uninstallAll();
  auto k = std::make_shared<FakeKernel>(3, std::vector<size_t>{2, 3});
  reg.installBackward("k|in:0", k, {2, 3}, {2, 3}, {1}, 2);
  std::mt19937 rng(2);
  Tensor g = hostTensor({2, 3}, rng, -1, 1), a = hostTensor({2, 3}, rng, -1, 1);
  CHECK(reg.hasBackwardKey("k|in:0") && !reg.hasBackwardKey("k|in:1"));
  CHECK(!reg.tryExecuteBackward("k|in:0", g, {a}).has_value());  // map index 1 out of range
  CHECK(reg.tryExecuteBackward("k|in:0", g, {a, a}).has_value());
  Tensor g2 = hostTensor({3, 3}, rng, -1, 1);
  CHECK(!reg.tryExecuteBackward("k|in:0", g2, {a, a}).has_value());  // grad shape mismatch
  reg.uninstallAll();
}

TEST(region_registry_cost_gating_and_masks, false) {
  auto& rr = RegionFusionRegistry::getInstance();
  rr.clear();
  CHECK(rr.installedCountNoLock() == 0 && !rr.mayMatchAsLastOp(op::ReLU));
  auto k = std::make_shared<FakeKernel>(3, std::vector<size_t>{2, 2});
  rr.installWithCost({op::MatMul, op::Add, op::ReLU}, k, {4, 4, 4}, {{2, 3}, {3, 2}});
  CHECK(rr.installedCountNoLock() == 1 && rr.mayMatchAsLastOp(op::ReLU) && !rr.mayMatchAsLastOp(op::Add));
  CHECK(rr.find(RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{2, 3}, {3, 2}})) != nullptr);
  rr.installWithCost({op::MatMul, op::ReLU}, k, {4, 4}, {{2, 3}});  // not worthwhile: inactive
  CHECK(rr.find(RegionFusionRegistry::regionKey({op::MatMul, op::ReLU}, {{2, 3}})) == nullptr);
  rr.installWithCost({op::Add, op::ReLU}, k, {4}, {});  // incomplete numels: inactive
  CHECK(rr.find(RollingHash::hashSequence({op::Add, op::ReLU})) == nullptr);
  rr.installFromCompiledKernel({op::Add, op::ReLU}, k);  // unmixed hash: reachable by matching
  auto prefix = RollingHash::computePrefixHashes({op::Mul, op::Add, op::ReLU});
  CHECK(rr.matchFromPosition(prefix, 1, {}) != nullptr && rr.matchFromPosition(prefix, 0, {}) == nullptr);
  rr.clear();
}

TEST(engine_lowers_graphs_onto_b200_kernels, false) {
  auto& eng = C3Engine::getInstance();
  eng.clearCache();
  auto k = std::dynamic_pointer_cast<CudaKernelBase>(eng.compile(regionGraph(128, 784, 256)));
  CHECK(k && k->describe().find("region") == 0);
  CHECK(eng.compile(regionGraph(128, 784, 256)).get() == k.get());  // cache hit
  CHECK(eng.getCacheStats().hits >= 1);
  // MatMul backward graphs: transposes fold into the GEMM
  TensorDesc g = TensorDesc::fromShape({8, 4}), a = TensorDesc::fromShape({8, 6}), b = TensorDesc::fromShape({6, 4});
  for (size_t i = 0; i < 2; ++i) {
    auto bg = C3BackwardCapture::getInstance().buildBackwardGraphForTypeAndIndex("10MatMulNode", i, g, {a, b});
    CHECK(bg.has_value());
    auto mk = std::dynamic_pointer_cast<CudaKernelBase>(eng.compile(bg->first));
    CHECK(mk && mk->describe().find(i == 0 ? "B^T" : "A^T") != std::string::npos);
    CHECK(bg->second == std::vector<size_t>{i == 0 ? 1u : 0u});
  }
  // ReLU backward, Add-backward SumReduce, Sigmoid backward (elementwise program)
  auto relu = C3BackwardCapture::getInstance().buildBackwardGraphForTypeAndIndex("8ReLUNode", 0, g, {g});
  CHECK(std::dynamic_pointer_cast<CudaKernelBase>(eng.compile(relu->first))->describe() == "relu_backward");
  auto add = C3BackwardCapture::getInstance().buildBackwardGraphForTypeAndIndex(
      "7AddNode", 1, g, {g, TensorDesc::fromShape({4})});
  CHECK(std::dynamic_pointer_cast<CudaKernelBase>(eng.compile(add->first))->describe() == "sum_reduce_axis0");
  auto sig = C3BackwardCapture::getInstance().buildBackwardGraphForTypeAndIndex("11SigmoidNode", 0, g, {g});
  CHECK(std::dynamic_pointer_cast<CudaKernelBase>(eng.compile(sig->first))->describe().find("elementwise") == 0);
  // identity (Add lhs grad) has nothing to compile
  auto ident = C3BackwardCapture::getInstance().buildBackwardGraphForTypeAndIndex("7AddNode", 0, g, {g, g});
  bool threw = false;
  try {
    eng.compile(ident->first);
  } catch (const std::exception&) {
    threw = true;
  }
  CHECK(threw && !eng.getLastCompileError().empty());
}

TEST(engine_async_dedup_and_timeout, false) {
  auto& eng = C3Engine::getInstance();
  eng.clearCache();
  Graph g = regionGraph(64, 64, 64);
  auto f1 = eng.compileAsync(g), f2 = eng.compileAsync(g);
  CHECK(f1.get() != nullptr && f2.get() == f1.get());
  // a failing compile yields nullptr through the future, no throw
  Graph empty;
  auto x = TensorDesc::fromShape({2});
  empty.markOutput(empty.addInput(x));
  CHECK(eng.compileAsync(empty).get() == nullptr);
  CHECK(eng.getCacheStats().async_failures >= 1);
}

TEST(hot_path_trigger_installs_region, false) {
  auto& hp = C3HotPathManager::instance();
  hp.clear();
  HotPathConfig cfg;
  cfg.hot_threshold = 3;
  hp.configure(cfg);
  RegionFusionRegistry::getInstance().clear();
  C3KernelRegistry::getInstance().uninstallAll();
  for (int i = 0; i < 3; ++i) {
    hp.recordCall(op::MatMul, DeviceType::kCUDA, {128, 784}, {784, 256});
    hp.recordCall(op::Add, DeviceType::kCUDA, {128, 256}, {256});
    hp.recordCall(op::ReLU, DeviceType::kCUDA, {128, 256});
  }
  hp.waitForPendingCompiles();
  auto* e = RegionFusionRegistry::getInstance().find(
      RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{128, 784}, {784, 256}}));
  CHECK(e != nullptr && e->cost.worthwhile && e->len == 3);
  CHECK(C3KernelRegistry::getInstance().fusedEntryCount() == 1);
  auto f = C3KernelRegistry::getInstance().findFusedKernelForSequence({op::MatMul, op::Add, op::ReLU},
                                                                      DeviceType::kCUDA, {128, 784});
  CHECK(f.has_value() && f->second.fused_pattern == "MatMul+Add+ReLU" && f->second.K == 784);
  CHECK(hp.getStats().compilations_triggered >= 1);
  // the graph built for the region has the reference's input order {X, B, b}
  C3HotPathManager::DispatchRecord r0{op::MatMul, {4, 3, 3, 2}, {4, 3}, {3, 2}, {}};
  C3HotPathManager::DispatchRecord r1{op::Add, {4, 2, 2}, {4, 2}, {2}, {}};
  C3HotPathManager::DispatchRecord r2{op::ReLU, {4, 2}, {4, 2}, {}, {}};
  Graph g = C3HotPathManager::buildFusedGraphForTest({r0, r1, r2}, "MatMul+Add+ReLU");
  CHECK(g.inputCount() == 3 && g.node(g.inputs()[2]).out_desc.shape == std::vector<size_t>{2});
  hp.shutdown();
  hp.clear();
}

TEST(backward_keys_and_disabled_device_path, false) {
  std::string key = C3BackwardCapture::makeBaseKey("8ReLUNode", {128, 256}, {{128, 256}});
  CHECK(key == "8ReLUNode|grad:128,256,|inputs:128,256,");
  CHECK(C3BackwardCapture::needsSumReduce({128, 256}, {256}) && !C3BackwardCapture::needsSumReduce({2, 3}, {2, 3}));
  CHECK(C3BackwardCapture::computeReduceAxis({128, 256}, {256}) == 0);
  CHECK(C3BackwardCapture::computeReduceAxis({128, 256}, {1, 256}) == 0);
  CHECK(C3BackwardCapture::supportsNodeType("10MatMulNode") && !C3BackwardCapture::supportsNodeType("Foo"));
}

TEST(fused_backward_sequence_detection, false) {
  auto& bc = C3BackwardCapture::getInstance();
  bc.clear();
  const std::vector<size_t> shp{32, 64};
  Tensor x(ShapeTag{}, shp, DType::kFloat, DeviceType::kCPU);
  const std::string sig = typeid(::SigmoidNode).name(), tanh_t = typeid(::TanhNode).name(),
                    mm = typeid(::MatMulNode).name();
  // backward order of y = sigmoid(tanh(x)): Sigmoid first, then Tanh
  bc.recordBackwardNode(sig, shp, shp, {x});
  bc.recordBackwardNode(tanh_t, shp, shp, {x});
  bc.recordBackwardNode(mm, shp, shp, {x});  // not elementwise: never enters the window
  bc.waitForPendingCompiles();
  const std::string key = C3BackwardCapture::makeFusedBackwardKey("Sigmoid+Tanh", shp, shp);
  CHECK(key == "backward_fused_Sigmoid+Tanh|g:32,64,|i:32,64,");
  CHECK(C3KernelRegistry::getInstance().hasBackwardKey(key));
  CHECK(bc.getStats().fusion_compile_count >= 1);
  CHECK(C3BackwardCapture::makeSequenceKey({sig, tanh_t, typeid(::ReLUNode).name()}) == "Sigmoid+Tanh+ReLU");
  CHECK(!C3BackwardCapture::isFusableSequence({sig}));
  CHECK(!C3BackwardCapture::isFusableSequence({sig, mm}));
  CHECK(C3BackwardCapture::isElementWiseBackward(typeid(::ExpNode).name()) &&
        !C3BackwardCapture::isElementWiseBackward(typeid(::AddNode).name()));
}

// Backward capture from several autograd threads at once: each records Sigmoid -> Tanh
// backward pairs of its own shape (one recording window for all threads) while fused-backward
// compiles run in the background, and probes the registry for its fused key. Checks: compiles
// finish, at least one thread's pair is installed under its exact key, and no probe sees a
// partial entry. Run under ThreadSanitizer too.
TEST(backward_capture_concurrent_recording, false) {
  auto& bc = C3BackwardCapture::getInstance();
  auto& reg = C3KernelRegistry::getInstance();
  bc.clear();
  reg.uninstallAll();
  const std::string sig = typeid(::SigmoidNode).name(), tanh_t = typeid(::TanhNode).name();
  constexpr int kThreads = 4, kRounds = 100;
  std::atomic<bool> go{false};
  std::vector<std::thread> threads;
  for (int t = 0; t < kThreads; ++t)
    threads.emplace_back([&, t] {
      while (!go.load()) std::this_thread::yield();
      const std::vector<size_t> shp{16 * static_cast<size_t>(t + 1), 64};
      Tensor x(ShapeTag{}, shp, DType::kFloat, DeviceType::kCPU);
      const std::string key = C3BackwardCapture::makeFusedBackwardKey("Sigmoid+Tanh", shp, shp);
      for (int i = 0; i < kRounds; ++i) {
        bc.recordBackwardNode(sig, shp, shp, {x});
        bc.recordBackwardNode(tanh_t, shp, shp, {x});
        (void)reg.hasBackwardKey(key);
        (void)bc.getStats();
      }
    });
  go.store(true);
  for (auto& th : threads) th.join();
  bc.waitForPendingCompiles();
  size_t installed = 0;
  for (int t = 0; t < kThreads; ++t) {
    const std::vector<size_t> shp{16 * static_cast<size_t>(t + 1), 64};
    installed += reg.hasBackwardKey(C3BackwardCapture::makeFusedBackwardKey("Sigmoid+Tanh", shp, shp));
  }
  CHECK(installed >= 1);
  CHECK(bc.getStats().fusion_compile_count >= 1);
  bc.clear();
  reg.uninstallAll();
}

// ============================================================================ GPU
TEST(gpu_region_fp32_is_bit_exact_through_registry, true) {
  // cfg1 layer shapes: the fp32 path reproduces the reference's loop arithmetic exactly.
  std::mt19937 rng(7);
  const size_t shapes[3][3] = {{128, 784, 256}, {128, 256, 128}, {128, 128, 10}};
  for (auto& s : shapes) {
    const size_t M = s[0], K = s[1], N = s[2];
    Tensor X = hostTensor({M, K}, rng, 0.f, 1.f), B = hostTensor({K, N}, rng, -0.1f, 0.1f),
           b = hostTensor({N}, rng, -0.1f, 0.1f);
    auto k = C3Engine::getInstance().compile(regionGraph(M, K, N));
    KernelShapeInfo info{{M, K}, {K, N}, {M, N}, true, M, K, N, "MatMul+Add+ReLU"};
    Tensor Y = C3KernelRegistry::getInstance().executeFusedWithInputs(k, {X, B, b}, info);
    CHECK(Y.defined() && Y.device() == DeviceType::kCPU && Y.shape() == std::vector<size_t>({M, N}));
    std::vector<float> ref(M * N), z(M * N);
    c3o_region_fwd(X.data_read<float>(), B.data_read<float>(), b.data_read<float>(), N, ref.data(), z.data(),
                   M, K, N, 0, 0, M, 4);
    CHECK(Y.defined() && std::memcmp(Y.data_read<float>(), ref.data(), M * N * 4) == 0);
  }
}

TEST(gpu_host_tensor_staging_round_trip, true) {
  // Host <-> device copies of a host framework's (pageable) tensors: large ones go through the
  // pinned staging pipeline in chunks (ragged last chunk here), small ones directly.
  for (size_t n : {size_t(3), size_t(1) << 20, (size_t(25) << 20) + 12345}) {
    Tensor h(ShapeTag{}, {n}, DType::kFloat, DeviceType::kCPU);
    for (size_t i = 0; i < n; ++i) h.data_write<float>()[i] = static_cast<float>((i * 2654435761u) % 1000003u);
    Tensor d = h.to(DeviceType::kCUDA);
    Tensor d2 = d.to(DeviceType::kCUDA);  // device -> device
    Tensor back = d2.to(DeviceType::kCPU);
    CHECK(back.numel() == n && std::memcmp(back.data_read<float>(), h.data_read<float>(), n * 4) == 0);
  }
}

TEST(gpu_backward_capture_relu_matmul_add, true) {
  std::mt19937 rng(9);
  const size_t M = 64, K = 96, N = 40;
  auto& bc = C3BackwardCapture::getInstance();
  Tensor x = hostTensor({M, N}, rng, -1, 1), grad = hostTensor({M, N}, rng, -1, 1);
  ::ReLUNode relu({x});
  CHECK(!bc.tryExecuteBackward(&relu, grad, {x}).has_value());  // first visit: miss + compile
  bc.waitForPendingCompiles();
  auto r = bc.tryExecuteBackward(&relu, grad, {x});
  CHECK(r.has_value() && r->size() == 1);
  std::vector<float> ref(M * N);
  c3o_relu_bwd(grad.data_read<float>(), x.data_read<float>(), ref.data(), M * N);
  CHECK(r && std::memcmp((*r)[0].data_read<float>(), ref.data(), M * N * 4) == 0);

  Tensor A = hostTensor({M, K}, rng, -1, 1), Bm = hostTensor({K, N}, rng, -1, 1);
  ::MatMulNode mm({A, Bm});
  CHECK(!bc.tryExecuteBackward(&mm, grad, {A, Bm}).has_value());
  bc.waitForPendingCompiles();
  CHECK(!bc.tryExecuteBackward(&mm, grad, {A, Bm}).has_value());  // second input compiles now
  bc.waitForPendingCompiles();
  auto g = bc.tryExecuteBackward(&mm, grad, {A, Bm});
  CHECK(g.has_value() && g->size() == 2);
  if (g) {
    std::vector<float> dA(M * K), dB(K * N);
    c3o_matmul(grad.data_read<float>(), Bm.data_read<float>(), dA.data(), M, N, K, 0, 112, nullptr, 0, 0, 0, M, 1);
    c3o_matmul(A.data_read<float>(), grad.data_read<float>(), dB.data(), K, M, N, 112, 0, nullptr, 0, 0, 0, K, 1);
    CHECK(std::memcmp((*g)[0].data_read<float>(), dA.data(), dA.size() * 4) == 0);
    CHECK(std::memcmp((*g)[1].data_read<float>(), dB.data(), dB.size() * 4) == 0);
  }

  Tensor bias = hostTensor({N}, rng, -1, 1);
  ::AddNode add({x, bias});
  CHECK(!bc.tryExecuteBackward(&add, grad, {x, bias}).has_value());
  bc.compileBackwardAsync(&add, grad);  // every input: lhs (identity, skipped) and rhs (SumReduce)
  bc.waitForPendingCompiles();
  // lhs gradient is the identity (never compiled), so the node stays on the host's path
  CHECK(!bc.tryExecuteBackward(&add, grad, {x, bias}).has_value());
  std::vector<float> db(N);
  c3o_sum_reduce(grad.data_read<float>(), db.data(), M, N, 0);
  auto key = C3BackwardCapture::makeBaseKey(typeid(add).name(), grad.sizes(), {x.sizes(), bias.sizes()}) + "|in:1";
  auto rb = C3KernelRegistry::getInstance().tryExecuteBackward(key, grad, {x, bias});
  CHECK(rb.has_value() && std::memcmp((*rb)[0].data_read<float>(), db.data(), N * 4) == 0);
}

TEST(gpu_region_bf16_device_tensors, true) {
  // bf16 device tensors take the tcgen05 path; compare with the fp32 oracle within 2e-2.
  const size_t M = 256, K = 512, N = 384;
  std::mt19937 rng(11);
  Tensor X = hostTensor({M, K}, rng, -1, 1), B = hostTensor({K, N}, rng, -0.05f, 0.05f),
         b = hostTensor({N}, rng, -0.1f, 0.1f);
  auto toBf16Dev = [](const Tensor& t) {
    Tensor d = t.to(DeviceType::kCUDA);
    Tensor o(ShapeTag{}, t.shape(), DType::kBF16, DeviceType::kCUDA);
    c3cu_convert(d.data(), C3CU_DTYPE_F32, o.data(), C3CU_DTYPE_BF16, t.numel(), ct::c3::cuda::currentStream());
    return o;
  };
  auto toF32Host = [](const Tensor& t) {
    Tensor f(ShapeTag{}, t.shape(), DType::kFloat, DeviceType::kCUDA);
    c3cu_convert(t.data(), C3CU_DTYPE_BF16, f.data(), C3CU_DTYPE_F32, t.numel(), ct::c3::cuda::currentStream());
    return f.to(DeviceType::kCPU);
  };
  Tensor Xd = toBf16Dev(X), Bd = toBf16Dev(B), bd = b.to(DeviceType::kCUDA);
  auto k = C3Engine::getInstance().compile(regionGraph(M, K, N));
  auto outs = k->execute({Xd, Bd, bd});
  CHECK(outs.size() == 2 && outs[0].device() == DeviceType::kCUDA && outs[0].dtype() == DType::kBF16);
  Tensor Xh = toF32Host(Xd), Bh = toF32Host(Bd), Y = toF32Host(outs[0]);
  std::vector<float> ref(M * N), z(M * N);
  c3o_region_fwd(Xh.data_read<float>(), Bh.data_read<float>(), b.data_read<float>(), N, ref.data(), z.data(), M, K,
                 N, 0, 0, M, 4);
  double max_err = 0, max_ref = 0;
  for (size_t i = 0; i < M * N; ++i) {
    max_err = std::max(max_err, (double)std::fabs(Y.data_read<float>()[i] - ref[i]));
    max_ref = std::max(max_ref, (double)std::fabs(ref[i]));
  }
  CHECK(max_err / max_ref <= 2e-2);
  uint32_t fault = 0;
  CHECK(c3cu_fault_status(&fault) == 0 && fault == 0);
}

TEST(gpu_fused_backward_chain_intercepts, true) {
  // y = Sigmoid(Tanh(Exp(x))): backward visits Sigmoid, Tanh, Exp. The recording window counts
  // a complete two-node chain and then restarts (src/C3/C3BackwardCapture.cpp:886-931), so the
  // compiled sequence is the pair Sigmoid+Tanh: the fused kernel runs once at Sigmoid, Tanh
  // receives its gradient from the intercept table (path A), and Exp stays on the host's path.
  auto& bc = C3BackwardCapture::getInstance();
  bc.clear();
  std::mt19937 rng(21);
  const size_t R = 64, C = 96, n = R * C;
  Tensor x0 = hostTensor({R, C}, rng, -1.5f, 1.5f);  // Exp input
  Tensor x1 = hostTensor({R, C}, rng, -2.f, 2.f);    // Tanh input
  Tensor x2 = hostTensor({R, C}, rng, -3.f, 3.f);    // Sigmoid input
  Tensor grad = hostTensor({R, C}, rng, -1.f, 1.f);
  auto exp_n = std::make_shared<::ExpNode>(std::vector<Tensor>{x0});
  auto tanh_n = std::make_shared<::TanhNode>(std::vector<Tensor>{x1});
  auto wrap = std::make_shared<::FactorNode>(std::vector<Tensor>{x1});
  wrap->setUpStreamNodes({exp_n});
  tanh_n->setUpStreamNodes({wrap});  // a wrapper between two elementwise nodes is skipped
  auto sig_n = std::make_shared<::SigmoidNode>(std::vector<Tensor>{x2});
  sig_n->setUpStreamNodes({tanh_n});
  for (auto* t : {typeid(::SigmoidNode).name(), typeid(::TanhNode).name(), typeid(::ExpNode).name()})
    bc.recordBackwardNode(t, {R, C}, {R, C}, {x0});
  bc.waitForPendingCompiles();
  auto g0 = bc.tryExecuteFusedBackward(sig_n.get(), grad, {x2});
  CHECK(g0.has_value());
  auto g1 = bc.tryExecuteFusedBackward(tanh_n.get(), grad, {x1});  // grad is ignored: intercepted
  auto g2 = bc.tryExecuteFusedBackward(exp_n.get(), grad, {x0});
  CHECK(g1.has_value() && !g2.has_value());
  std::vector<float> r0(n), r1(n), r2(n);
  const int ops[3] = {C3CU_BW_SIGMOID, C3CU_BW_TANH, C3CU_BW_EXP};
  const float* xs[3] = {x2.data_read<float>(), x1.data_read<float>(), x0.data_read<float>()};
  float* outs[3] = {r0.data(), r1.data(), r2.data()};
  c3o_backward_chain(ops, 3, grad.data_read<float>(), xs, outs, n);
  auto close = [&](const Tensor& t, const std::vector<float>& ref) {
    double worst = 0, scale = 0;
    for (size_t i = 0; i < n; ++i) {
      worst = std::max(worst, (double)std::fabs(t.data_read<float>()[i] - ref[i]));
      scale = std::max(scale, (double)std::fabs(ref[i]));
    }
    return worst <= 1e-5 * scale;
  };
  CHECK(g0 && close(*g0, r0));
  CHECK(g1 && close(*g1, r1));
  CHECK(bc.getStats().fusion_hit_count >= 2);
  CHECK(C3KernelRegistry::getInstance().hasBackwardKey(
      C3BackwardCapture::makeFusedBackwardKey("Sigmoid+Tanh", {R, C}, {R, C})));
  CHECK(!C3KernelRegistry::getInstance().hasBackwardKey(
      C3BackwardCapture::makeFusedBackwardKey("Sigmoid+Tanh+Exp", {R, C}, {R, C})));
  // a node outside any compiled chain misses once, then is remembered as a miss
  auto lone = std::make_shared<::NegNode>(std::vector<Tensor>{x0});
  CHECK(!bc.tryExecuteFusedBackward(lone.get(), grad, {x0}).has_value());
  CHECK(!bc.tryExecuteFusedBackward(lone.get(), grad, {x0}).has_value());
  bc.clearInterceptedState();
  uint32_t fault = 0;
  CHECK(c3cu_fault_status(&fault) == 0 && fault == 0);
}

TEST(gpu_two_tier_matmul_tuned_tier, true) {
  // opt 2 (precompiled) and opt 4 (tuned) bind the same GEMM; the first run of the opt-4
  // kernel times the variants for its shape and installs the fastest, the registry keeps
  // the higher level, and both tiers agree to bf16 rounding.
  c3cu_gemm_tune_clear();
  const size_t M = 512, K = 1024, N = 768;
  std::mt19937 rng(31);
  Tensor A = hostTensor({M, K}, rng, -1, 1), B = hostTensor({K, N}, rng, -0.05f, 0.05f);
  auto bf16Dev = [](const Tensor& t) {
    Tensor d = t.to(DeviceType::kCUDA);
    Tensor o(ShapeTag{}, t.shape(), DType::kBF16, DeviceType::kCUDA);
    c3cu_convert(d.data(), C3CU_DTYPE_F32, o.data(), C3CU_DTYPE_BF16, t.numel(), ct::c3::cuda::currentStream());
    return o;
  };
  Tensor Ad = bf16Dev(A), Bd = bf16Dev(B);
  Graph g;
  auto a = TensorDesc::fromShape({M, K}), b = TensorDesc::fromShape({K, N}), o = TensorDesc::fromShape({M, N});
  const size_t ai = g.addInput(a), bi = g.addInput(b);
  g.markOutput(g.addNode(c3::MatMulNode{a, b}, {ai, bi}, o));
  c3::CompileOptions fast, tuned;
  fast.opt_level = 2;
  tuned.opt_level = 4;
  auto k2 = C3Engine::getInstance().compile(g, fast);
  auto k4 = C3Engine::getInstance().compile(g, tuned);
  CHECK(k2 && k4 && k2->optLevel() == 2 && k4->optLevel() == 4);
  auto& reg = C3KernelRegistry::getInstance();
  reg.uninstallAll();
  KernelShapeInfo info{{M, K}, {K, N}, {M, N}, true, M, K, N, ""};
  reg.install(op::MatMul, DeviceType::kCUDA, k4, info);
  reg.install(op::MatMul, DeviceType::kCUDA, k2, info);  // lower level: the tuned tier stays
  auto y4 = k4->execute({Ad, Bd});
  int variant = -1;
  // B [K, N] is read MN-major (b_mn = 1) by the bf16 GEMM, A K-major; bf16 output
  CHECK(c3cu_gemm_tune_get(M, N, K, 0, 1, C3CU_EPI_STORE_BF16, &variant) == 0 && variant >= 0 && variant <= 2);
  auto y2 = k2->execute({Ad, Bd});
  auto toF32 = [](const Tensor& t) {
    Tensor f(ShapeTag{}, t.shape(), DType::kFloat, DeviceType::kCUDA);
    c3cu_convert(t.data(), C3CU_DTYPE_BF16, f.data(), C3CU_DTYPE_F32, t.numel(), ct::c3::cuda::currentStream());
    return f.to(DeviceType::kCPU);
  };
  Tensor h4 = toF32(y4[0]), h2 = toF32(y2[0]);
  double worst = 0, scale = 0;
  for (size_t i = 0; i < M * N; ++i) {
    worst = std::max(worst, (double)std::fabs(h4.data_read<float>()[i] - h2.data_read<float>()[i]));
    scale = std::max(scale, (double)std::fabs(h2.data_read<float>()[i]));
  }
  CHECK(worst <= 2e-2 * scale);
  reg.uninstallAll();
  c3cu_gemm_tune_clear();
  uint32_t fault = 0;
  CHECK(c3cu_fault_status(&fault) == 0 && fault == 0);
}

int main(int argc, char** argv) {
  const bool gpu = argc > 1 && std::string(argv[1]) == "--gpu";
  // --only NAME: run that test alone (e.g. the concurrency test under ThreadSanitizer)
  const std::string only = (argc > 3 && std::string(argv[2]) == "--only") ? argv[3] : "";
  int ran = 0;
  for (auto& t : registry()) {
    if (t.gpu != gpu || (!only.empty() && only != t.name)) continue;
    const int before = g_failures;
    try {
      t.fn();
    } catch (const std::exception& e) {
      ++g_failures;
      std::fprintf(stderr, "  exception: %s\n", e.what());
    }
    std::printf("%s %s\n", g_failures == before ? "PASS" : "FAIL", t.name);
    ++ran;
  }
  shutdownAll();
  std::printf("%d tests, %d checks, %d failures\n", ran, g_checks, g_failures);
  return g_failures == 0 ? 0 : 1;
}
