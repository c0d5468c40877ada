// Drives the C++ mirror of the C3 API the way a host framework does, and prints one JSON object.
//
//   api_drive mlp [steps]            the cfg1 MLP training loop (784 -> 256 -> 128 -> 10, batch 128,
//                                    fp32 host tensors, softmax cross-entropy, SGD lr 0.01). Every op
//                                    is recorded with C3HotPathManager::recordCall; the hidden
//                                    layers' MatMul+Add+ReLU run through RegionFusionRegistry::find
//                                    -> C3KernelRegistry::executeFusedWithInputs once installed, the
//                                    output layer's MatMul and Add through C3KernelRegistry::tryExecute,
//                                    and every autograd node's backward through
//                                    C3BackwardCapture::tryExecuteBackward. Misses run the host's
//                                    own eager ops. The same loop runs beside it on the oracle
//                                    (liboracle.so, test infrastructure) with the same op
//                                    decomposition; parameters, logits and loss are compared bit for bit.
//   api_drive region [M K N iters]   the cfg2 region (bf16 X [M,K], B [K,N], fp32 b [N]) through
//                                    executeFusedWithInputs with host tensors: each call copies its
//                                    inputs to the GPU and its outputs (Y, ReLU mask) back, as the
//                                    reference's CompiledKernel::execute contract has it. Timed with
//                                    B on the host (every call uploads it) and with B resident on the
//                                    device (as a training loop keeps its weights).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "AutoGrad/Node.h"
#include "C3/C3BackwardCapture.h"
#include "C3/C3Cleanup.h"
#include "C3/C3Engine.h"
#include "C3/C3HotPathManager.h"
#include "C3/C3KernelRegistry.h"
#include "C3/CudaRuntime.h"
#include "C3/RegionFusion.h"
#include "c3cu.h"

extern "C" {
void c3o_region_fwd(const float* X, const float* B, const float* b, size_t b_numel, float* out, float* z,
                    size_t M, size_t K, size_t N, int transB, size_t r0, size_t r1, int threads);
void c3o_matmul(const float* A, const float* B, float* out, size_t M, size_t K, size_t N, int transA,
                int transB, const float* bias, size_t bias_numel, int act, size_t r0, size_t r1, int threads);
void c3o_relu_bwd(const float* grad, const float* x, float* out, size_t n);
void c3o_sum_reduce(const float* in, float* out, size_t M, size_t N, int axis);
void c3o_softmax_ce(const float* z, const int32_t* y, float* loss, float* dz, size_t B, size_t C);
void c3o_sgd(float* p, const float* g, size_t n, float lr);
}

namespace c3 = ct::c3;
using Clock = std::chrono::steady_clock;

static double seconds(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double>(b - a).count();
}

static Tensor host(const std::vector<size_t>& shape, DType dt = DType::kFloat) {
  return Tensor(ShapeTag{}, shape, dt, DeviceType::kCPU);
}

// ------------------------------------------------------------------ the host's eager ops
// The host framework's own CPU kernels, used on a miss; they follow the oracle's arithmetic.
static Tensor hostMatMul(const Tensor& A, const Tensor& B) {
  const size_t M = A.shape()[0], K = A.shape()[1], N = B.shape()[1];
  Tensor out = host({M, N});
  c3o_matmul(A.data_read<float>(), B.data_read<float>(), out.data_write<float>(), M, K, N, 0, 0, nullptr, 0, 0,
             0, M, 1);
  return out;
}

static Tensor hostAddBias(const Tensor& T, const Tensor& b) {
  Tensor out = host(T.shape());
  const size_t n = T.numel(), nb = b.numel();
  for (size_t i = 0; i < n; ++i) out.data_write<float>()[i] = T.data_read<float>()[i] + b.data_read<float>()[i % nb];
  return out;
}

static Tensor hostReLU(const Tensor& z) {
  Tensor out = host(z.shape());
  for (size_t i = 0; i < z.numel(); ++i) out.data_write<float>()[i] = std::fmax(z.data_read<float>()[i], 0.f);
  return out;
}

// ------------------------------------------------------------------ cfg1 MLP through the API
namespace mlp {

constexpr size_t kB = 128, kD0 = 784, kD1 = 256, kD2 = 128, kD3 = 10;
constexpr float kLr = 0.01f;

struct Params {
  Tensor W[3], b[3];
};

Params init(uint32_t seed) {
  std::mt19937 rng(seed);
  const size_t dims[4] = {kD0, kD1, kD2, kD3};
  Params p;
  for (int l = 0; l < 3; ++l) {
    const float bound = std::sqrt(6.0f / static_cast<float>(dims[l]));
    std::uniform_real_distribution<float> u(-bound, bound);
    p.W[l] = host({dims[l], dims[l + 1]});
    for (size_t i = 0; i < p.W[l].numel(); ++i) p.W[l].data_write<float>()[i] = u(rng);
    p.b[l] = host({dims[l + 1]});
    std::memset(p.b[l].data_write<float>(), 0, dims[l + 1] * 4);
  }
  return p;
}

void batch(uint32_t seed, Tensor& x, std::vector<int32_t>& y) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> u(0.f, 1.f);
  std::uniform_int_distribution<int32_t> c(0, static_cast<int32_t>(kD3) - 1);
  x = host({kB, kD0});
  for (size_t i = 0; i < x.numel(); ++i) x.data_write<float>()[i] = u(rng);
  y.resize(kB);
  for (auto& v : y) v = c(rng);
}

struct Counters {
  size_t region_hits = 0, region_misses = 0, single_hits = 0, single_misses = 0, bw_hits = 0, bw_misses = 0;
};

// One step of the host framework: dispatch through C3, fall back to its eager ops on a miss.
// Returns the loss; writes the logits to `logits`.
float apiStep(Params& p, const Tensor& x, const std::vector<int32_t>& y, Counters& cnt, Tensor& logits) {
  auto& hp = c3::C3HotPathManager::instance();
  auto& rf = c3::RegionFusionRegistry::getInstance();
  auto& kr = c3::C3KernelRegistry::getInstance();
  auto& bc = c3::C3BackwardCapture::getInstance();
  const size_t dims[4] = {kD0, kD1, kD2, kD3};
  Tensor a[3];  // a[0] = x, a[1], a[2] = hidden activations
  Tensor T[3], Z[3];
  a[0] = x;
  std::shared_ptr<::MatMulNode> mm[3];
  std::shared_ptr<::AddNode> add[3];
  std::shared_ptr<::ReLUNode> relu[2];
  for (int l = 0; l < 3; ++l) {
    const size_t K = dims[l], N = dims[l + 1];
    hp.recordCall(op::MatMul, DeviceType::kCPU, {kB, K}, {K, N});
    hp.recordCall(op::Add, DeviceType::kCPU, {kB, N}, {N});
    if (l < 2) hp.recordCall(op::ReLU, DeviceType::kCPU, {kB, N});
    Tensor out;
    if (l < 2) {
      // the region: find(rolling hash ^ first-input shape key) -> executeFusedWithInputs
      c3::RegionEntry* e = rf.find(c3::RegionFusionRegistry::regionKey({op::MatMul, op::Add, op::ReLU}, {{kB, K}, {K, N}}));
      if (e != nullptr && e->kernel) {
        c3::KernelShapeInfo info{{kB, K}, {K, N}, {kB, N}, true, kB, K, N, "MatMul+Add+ReLU"};
        out = kr.executeFusedWithInputs(e->kernel, {a[l], p.W[l], p.b[l]}, info);
      }
      if (out.defined()) {
        ++cnt.region_hits;
      } else {
        ++cnt.region_misses;
        T[l] = hostMatMul(a[l], p.W[l]);
        Z[l] = hostAddBias(T[l], p.b[l]);
        out = hostReLU(Z[l]);
      }
      // autograd nodes. The ReLU node keeps its output: relu'(z) = [z > 0] = [relu(z) > 0], so
      // Gt(out, 0) * grad is the same gradient bit for bit, and the fused region need not
      // materialise its pre-activation.
      mm[l] = std::make_shared<::MatMulNode>(std::vector<Tensor>{a[l], p.W[l]});
      add[l] = std::make_shared<::AddNode>(std::vector<Tensor>{Tensor(ShapeTag{}, {kB, N}), p.b[l]});
      relu[l] = std::make_shared<::ReLUNode>(std::vector<Tensor>{out});
      a[l + 1] = out;
    } else {
      auto t = kr.tryExecute(op::MatMul, a[l], p.W[l]);
      if (t) ++cnt.single_hits; else ++cnt.single_misses;
      T[l] = t ? *t : hostMatMul(a[l], p.W[l]);
      auto z = kr.tryExecute(op::Add, T[l], p.b[l]);
      if (z) ++cnt.single_hits; else ++cnt.single_misses;
      Z[l] = z ? *z : hostAddBias(T[l], p.b[l]);
      mm[l] = std::make_shared<::MatMulNode>(std::vector<Tensor>{a[l], p.W[l]});
      add[l] = std::make_shared<::AddNode>(std::vector<Tensor>{T[l], p.b[l]});
    }
  }
  logits = Z[2];
  // loss (host framework)
  Tensor dz = host({kB, kD3});
  float loss = 0.f;
  c3o_softmax_ce(logits.data_read<float>(), y.data(), &loss, dz.data_write<float>(), kB, kD3);
  // backward: output layer first, then the hidden layers
  Tensor grad = dz, dW[3], db[3];
  for (int l = 2; l >= 0; --l) {
    const size_t K = dims[l], N = dims[l + 1];
    if (l < 2) {  // ReLU
      auto r = bc.tryExecuteBackward(relu[l].get(), grad, relu[l]->getInputs());
      if (r) {
        ++cnt.bw_hits;
        grad = (*r)[0];
      } else {
        ++cnt.bw_misses;
        Tensor g = host(grad.shape());
        c3o_relu_bwd(grad.data_read<float>(), relu[l]->getInputs()[0].data_read<float>(), g.data_write<float>(),
                     grad.numel());
        grad = g;
      }
    }
    // Add (T + b): the lhs gradient is the identity, which the reference never compiles, so the
    // node runs on the host: dT = grad, db = column sums of grad
    {
      auto r = bc.tryExecuteBackward(add[l].get(), grad, add[l]->getInputs());
      if (r && r->size() == 2) {
        ++cnt.bw_hits;
        db[l] = (*r)[1];
      } else {
        ++cnt.bw_misses;
        db[l] = host({N});
        c3o_sum_reduce(grad.data_read<float>(), db[l].data_write<float>(), kB, N, 0);
      }
    }
    // MatMul (a @ W): dA = grad W^T, dW = a^T grad
    auto r = bc.tryExecuteBackward(mm[l].get(), grad, mm[l]->getInputs());
    Tensor dA;
    if (r && r->size() == 2) {
      ++cnt.bw_hits;
      dA = (*r)[0];
      dW[l] = (*r)[1];
    } else {
      ++cnt.bw_misses;
      dA = host({kB, K});
      dW[l] = host({K, N});
      c3o_matmul(grad.data_read<float>(), p.W[l].data_read<float>(), dA.data_write<float>(), kB, N, K, 0, 112,
                 nullptr, 0, 0, 0, kB, 1);
      c3o_matmul(mm[l]->getInputs()[0].data_read<float>(), grad.data_read<float>(), dW[l].data_write<float>(), K,
                 kB, N, 112, 0, nullptr, 0, 0, 0, K, 1);
    }
    grad = dA;
  }
  bc.clearInterceptedState();
  // SGD (host framework)
  for (int l = 0; l < 3; ++l) {
    c3o_sgd(p.W[l].data_write<float>(), dW[l].data_read<float>(), p.W[l].numel(), kLr);
    c3o_sgd(p.b[l].data_write<float>(), db[l].data_read<float>(), p.b[l].numel(), kLr);
  }
  return loss;
}

// The same step on the oracle only, with the same op decomposition (region for the hidden
// layers, MatMul then Add for the output layer).
float oracleStep(Params& p, const Tensor& x, const std::vector<int32_t>& y, Tensor& logits) {
  const size_t dims[4] = {kD0, kD1, kD2, kD3};
  std::vector<float> act[3];
  act[0].assign(x.data_read<float>(), x.data_read<float>() + x.numel());
  std::vector<float> zpre[3];
  for (int l = 0; l < 2; ++l) {
    const size_t K = dims[l], N = dims[l + 1];
    act[l + 1].resize(kB * N);
    zpre[l].resize(kB * N);
    c3o_region_fwd(act[l].data(), p.W[l].data_read<float>(), p.b[l].data_read<float>(), N, act[l + 1].data(),
                   zpre[l].data(), kB, K, N, 0, 0, kB, 1);
  }
  std::vector<float> T3(kB * kD3);
  c3o_matmul(act[2].data(), p.W[2].data_read<float>(), T3.data(), kB, kD2, kD3, 0, 0, nullptr, 0, 0, 0, kB, 1);
  logits = host({kB, kD3});
  for (size_t i = 0; i < kB * kD3; ++i) logits.data_write<float>()[i] = T3[i] + p.b[2].data_read<float>()[i % kD3];
  std::vector<float> grad(kB * kD3);
  float loss = 0.f;
  c3o_softmax_ce(logits.data_read<float>(), y.data(), &loss, grad.data(), kB, kD3);
  std::vector<float> dW[3], db[3];
  for (int l = 2; l >= 0; --l) {
    const size_t K = dims[l], N = dims[l + 1];
    if (l < 2) {
      std::vector<float> g(kB * N);
      c3o_relu_bwd(grad.data(), act[l + 1].data(), g.data(), kB * N);
      grad.swap(g);
    }
    db[l].resize(N);
    c3o_sum_reduce(grad.data(), db[l].data(), kB, N, 0);
    std::vector<float> dA(kB * K);
    dW[l].resize(K * N);
    c3o_matmul(grad.data(), p.W[l].data_read<float>(), dA.data(), kB, N, K, 0, 112, nullptr, 0, 0, 0, kB, 1);
    c3o_matmul(act[l].data(), grad.data(), dW[l].data(), K, kB, N, 112, 0, nullptr, 0, 0, 0, K, 1);
    grad.swap(dA);
  }
  for (int l = 0; l < 3; ++l) {
    c3o_sgd(p.W[l].data_write<float>(), dW[l].data(), p.W[l].numel(), kLr);
    c3o_sgd(p.b[l].data_write<float>(), db[l].data(), p.b[l].numel(), kLr);
  }
  return loss;
}

bool sameBits(const Tensor& a, const Tensor& b) {
  return a.numel() == b.numel() && std::memcmp(a.data_read<float>(), b.data_read<float>(), a.numel() * 4) == 0;
}

int run(int steps) {
  auto& hp = c3::C3HotPathManager::instance();
  auto& bc = c3::C3BackwardCapture::getInstance();
  c3::HotPathConfig cfg;  // the reference's defaults: threshold 5, cooldown 60 s
  hp.configure(cfg);
  Params api = init(1234), ref = init(1234);
  Counters warm, timed;
  bool logits_exact = true, loss_exact = true;
  Tensor x, la, lr;
  std::vector<int32_t> y;
  // warm-up: the first cfg.hot_threshold steps record the dispatches; compiles run in the
  // background and are awaited so that the timed steps find every kernel installed
  const int warm_steps = static_cast<int>(cfg.hot_threshold) + 2;
  for (int s = 0; s < warm_steps; ++s) {
    batch(100 + s, x, y);
    const float l1 = apiStep(api, x, y, warm, la);
    const float l2 = oracleStep(ref, x, y, lr);
    logits_exact = logits_exact && sameBits(la, lr);
    loss_exact = loss_exact && std::memcmp(&l1, &l2, 4) == 0;
    hp.waitForPendingCompiles();
    bc.waitForPendingCompiles();
  }
  double api_s = 0, ora_s = 0;
  float last_loss = 0;
  for (int s = 0; s < steps; ++s) {
    batch(1000 + s, x, y);
    const auto t0 = Clock::now();
    const float l1 = apiStep(api, x, y, timed, la);
    const auto t1 = Clock::now();
    const float l2 = oracleStep(ref, x, y, lr);
    const auto t2 = Clock::now();
    api_s += seconds(t0, t1);
    ora_s += seconds(t1, t2);
    logits_exact = logits_exact && sameBits(la, lr);
    loss_exact = loss_exact && std::memcmp(&l1, &l2, 4) == 0;
    last_loss = l1;
  }
  bool params_exact = true;
  for (int l = 0; l < 3; ++l) params_exact = params_exact && sameBits(api.W[l], ref.W[l]) && sameBits(api.b[l], ref.b[l]);
  uint32_t fault = 0;
  const int frc = c3cu_fault_status(&fault);
  const auto ks = c3::C3KernelRegistry::getInstance().getStats();
  const auto bs = bc.getStats();
  std::printf(
      "{\"mode\": \"mlp\", \"steps\": %d, \"warmup_steps\": %d, \"us_per_step\": %.3f, \"oracle_us_per_step\": %.3f, "
      "\"timed\": {\"region_hits\": %zu, \"region_misses\": %zu, \"single_op_hits\": %zu, \"single_op_misses\": %zu, "
      "\"bw_hits\": %zu, \"bw_misses\": %zu}, "
      "\"registry\": {\"fused_hit_count\": %zu, \"hit_count\": %zu, \"backward_cache_hits\": %zu, "
      "\"backward_cache_misses\": %zu, \"compilations\": %zu}, "
      "\"loss\": %.7g, \"logits_bit_exact\": %s, \"loss_bit_exact\": %s, \"params_bit_exact\": %s, \"fault\": %u, "
      "\"path\": \"C3HotPathManager::recordCall -> RegionFusionRegistry::find -> "
      "C3KernelRegistry::executeFusedWithInputs / tryExecute; C3BackwardCapture::tryExecuteBackward; fp32 host "
      "tensors staged per call\"}\n",
      steps, warm_steps, api_s / steps * 1e6, ora_s / steps * 1e6, timed.region_hits, timed.region_misses,
      timed.single_hits, timed.single_misses, timed.bw_hits, timed.bw_misses, ks.fused_hit_count, ks.hit_count,
      bs.cache_hit_count, bs.cache_miss_count, hp.getStats().compilations_triggered, last_loss,
      logits_exact ? "true" : "false", loss_exact ? "true" : "false", params_exact ? "true" : "false", fault);
  const bool ok = logits_exact && loss_exact && params_exact && frc == 0 && fault == 0 &&
                  timed.region_misses == 0 && timed.region_hits == static_cast<size_t>(2 * steps);
  return ok ? 0 : 1;
}

}  // namespace mlp

// ------------------------------------------------------------------ cfg2 region, host tensors
namespace region {

uint16_t toBf16(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

float fromBf16(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

Tensor randomBf16(const std::vector<size_t>& shape, std::mt19937& rng, float stddev) {
  Tensor t = host(shape, DType::kBF16);
  std::normal_distribution<float> d(0.f, stddev);
  uint16_t* p = t.data_write<uint16_t>();
  for (size_t i = 0; i < t.numel(); ++i) p[i] = toBf16(d(rng));
  return t;
}

int run(size_t M, size_t K, size_t N, int iters) {
  std::mt19937 rng(2);
  Tensor X = randomBf16({M, K}, rng, 1.0f), B = randomBf16({K, N}, rng, 0.02f);
  Tensor b = host({N});
  std::normal_distribution<float> d(0.f, 0.01f);
  for (size_t i = 0; i < N; ++i) b.data_write<float>()[i] = d(rng);
  c3::Graph g;
  auto xd = c3::TensorDesc::fromShape({M, K}), bd = c3::TensorDesc::fromShape({K, N}),
       od = c3::TensorDesc::fromShape({M, N}), biasd = c3::TensorDesc::fromShape({N});
  const size_t xi = g.addInput(xd), bi = g.addInput(bd), ci = g.addInput(biasd);
  const size_t mmn = g.addNode(c3::MatMulNode{xd, bd}, {xi, bi}, od);
  const size_t addn = g.addNode(c3::AddNode{od, biasd}, {mmn, ci}, od);
  g.markOutput(g.addNode(c3::ReLUNode{od}, {addn}, od));
  auto kernel = c3::C3Engine::getInstance().compile(g);
  c3::KernelShapeInfo info{{M, K}, {K, N}, {M, N}, true, M, K, N, "MatMul+Add+ReLU"};
  auto& kr = c3::C3KernelRegistry::getInstance();
  const double flop = 2.0 * M * N * K;
  const double up_all = M * K * 2.0 + K * N * 2.0 + N * 4.0, up_x = M * K * 2.0 + N * 4.0;
  const double down = M * N * 2.0;  // Y bf16 (the graph output executeFusedWithInputs returns)
  auto timeIt = [&](const Tensor& Bin, Tensor& Y) {
    for (int i = 0; i < 2; ++i) Y = kr.executeFusedWithInputs(kernel, {X, Bin, b}, info);
    const auto t0 = Clock::now();
    for (int i = 0; i < iters; ++i) Y = kr.executeFusedWithInputs(kernel, {X, Bin, b}, info);
    return seconds(t0, Clock::now()) / iters;
  };
  Tensor Y1, Y2;
  const double t_host = timeIt(B, Y1);
  Tensor Bdev = B.to(DeviceType::kCUDA);
  const double t_res = timeIt(Bdev, Y2);
  // sampled rows against the oracle on the bf16-rounded inputs
  std::vector<float> Bf(K * N), xr(K), yr(N), zr(N);
  for (size_t i = 0; i < K * N; ++i) Bf[i] = fromBf16(B.data_read<uint16_t>()[i]);
  double max_err = 0, max_ref = 0;
  bool same = Y1.defined() && Y2.defined() &&
              std::memcmp(Y1.data_read<uint16_t>(), Y2.data_read<uint16_t>(), M * N * 2) == 0;
  const size_t row_step = std::max<size_t>(1, M / 16);
  for (size_t r = 0; r < M && Y1.defined(); r += row_step) {
    for (size_t k = 0; k < K; ++k) xr[k] = fromBf16(X.data_read<uint16_t>()[r * K + k]);
    c3o_region_fwd(xr.data(), Bf.data(), b.data_read<float>(), N, yr.data(), zr.data(), 1, K, N, 0, 0, 1, 1);
    for (size_t j = 0; j < N; ++j) {
      max_err = std::max(max_err, (double)std::fabs(fromBf16(Y1.data_read<uint16_t>()[r * N + j]) - yr[j]));
      max_ref = std::max(max_ref, (double)std::fabs(yr[j]));
    }
  }
  const double rel = max_ref > 0 ? max_err / max_ref : 1.0;
  uint32_t fault = 0;
  const int frc = c3cu_fault_status(&fault);
  std::printf(
      "{\"mode\": \"region\", \"M\": %zu, \"K\": %zu, \"N\": %zu, \"iters\": %d, "
      "\"host_weights\": {\"ms_per_call\": %.4f, \"tflops\": %.2f, \"h2d_bytes\": %.0f, \"d2h_bytes\": %.0f, "
      "\"gbs\": %.2f}, "
      "\"resident_weights\": {\"ms_per_call\": %.4f, \"tflops\": %.2f, \"h2d_bytes\": %.0f, \"d2h_bytes\": %.0f, "
      "\"gbs\": %.2f}, "
      "\"parity\": {\"rows_checked\": 16, \"max_rel\": %.3e, \"tol\": 2e-2, \"same_bits_both_ways\": %s}, "
      "\"fault\": %u, \"path\": \"C3Engine::compile -> C3KernelRegistry::executeFusedWithInputs -> "
      "CudaRegionKernel::execute (host tensors: pageable copies in and out, synchronous per call)\"}\n",
      M, K, N, iters, t_host * 1e3, flop / t_host / 1e12, up_all, down, (up_all + down) / t_host / 1e9,
      t_res * 1e3, flop / t_res / 1e12, up_x, down, (up_x + down) / t_res / 1e9, rel, same ? "true" : "false", fault);
  return (rel <= 2e-2 && same && frc == 0 && fault == 0) ? 0 : 1;
}

}  // namespace region

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "mlp";
  int rc = 2;
  try {
    if (mode == "mlp") {
      rc = mlp::run(argc > 2 ? std::atoi(argv[2]) : 50);
    } else if (mode == "region") {
      const size_t M = argc > 2 ? std::strtoull(argv[2], nullptr, 10) : 8192;
      const size_t K = argc > 3 ? std::strtoull(argv[3], nullptr, 10) : 4096;
      const size_t N = argc > 4 ? std::strtoull(argv[4], nullptr, 10) : 4096;
      rc = region::run(M, K, N, argc > 5 ? std::atoi(argv[5]) : 10);
    } else {
      std::fprintf(stderr, "usage: api_drive mlp [steps] | region [M K N iters]\n");
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "api_drive: %s\n", e.what());
    rc = 3;
  }
  c3::shutdownAll();
  return rc;
}
