// C-ABI entry points of the tcgen05 GEMM family (include/c3cu.h): the fused
// Linear+bias+ReLU forward, the dX / dW backward GEMMs and the general bf16 GEMM.
#include <atomic>
#include <map>
#include <tuple>
#include <mutex>
#include <utility>

#include "gemm2_tcgen05.cuh"
#include "gemm_tcgen05.cuh"
#include "host_util.h"

C3CU_FAULT_ACCESSORS(gemm)

namespace c3cu {
namespace {

using gemm::Params;

// Upper bound on the persistent GEMM's CTAs (0 = one per SM). Lowering it leaves SMs free
// for a collective that runs concurrently (e.g. an all-reduce overlapped with the dX GEMM).
// Per host thread: a cap set around one launch never reaches GEMMs other threads launch.
thread_local int g_max_ctas = 0;

// Per-shape variants chosen by a tuner (c3cu_gemm_tune_set); they take precedence over
// g_variant for an exact (M, N, K, majors, epilogue) match.
struct TuneKey {
  int64_t M, N, K;
  int a_mn, b_mn, epi;
  bool operator<(const TuneKey& o) const {
    return std::tie(M, N, K, a_mn, b_mn, epi) < std::tie(o.M, o.N, o.K, o.a_mn, o.b_mn, o.epi);
  }
};
std::mutex g_tune_mu;
std::map<TuneKey, int> g_tune;

// Kernel variant: 0 = automatic (the CTA-pair kernel whenever M spans at least two 128-row
// halves, with the split-K tail), 1 = single-CTA kernel only, 2 = CTA-pair kernel whenever it
// applies, without the split-K tail.
std::atomic<int> g_variant{0};

// Co-resident clusters of two CTAs for a kernel (cached per device and kernel).
template <class Kern>
int max_pair_clusters(Kern kern, uint32_t smem_bytes, int threads) {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int have = cached[dev].load(std::memory_order_relaxed);
  if (have > 0) return have;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Split-tile workspace of the CTA-pair kernel, one per (device, stream) so that kernels on
// different streams never share tickets: fp32 partials for `kSplitMax` shared tiles x 2 CTAs
// x 128 x 256 (a slot per cluster boundary, at most one per cluster), then per-warp tickets
// and ready words (zeroed once; every launch leaves them zero).
constexpr int kSplitMax = 80;
constexpr size_t kSplitPartialFloats = static_cast<size_t>(kSplitMax) * 2 * gemm2::HM * gemm2::TN;
constexpr size_t kSplitWords = static_cast<size_t>(kSplitMax) * 2 * gemm2::kEpiWarps;
constexpr size_t kSplitWsBytes = kSplitPartialFloats * 4 + 2 * kSplitWords * 4;

// Limit on a split tile's wait for its partner's partial (c3cu_set_split_wait_ns).
std::atomic<uint64_t> g_split_wait_ns{C3CU_WAIT_LIMIT_NS};

// Bumped by gemm_invalidate_split_workspaces (after a recorded fault): a workspace cleared
// under an older generation is cleared again before its next launch.
std::atomic<uint32_t> g_split_generation{0};

struct SplitWs {
  void* ws;
  uint32_t generation;
};

int split_workspace(cudaStream_t stream, float** partial, uint32_t** tickets, uint32_t** ready) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, SplitWs> pool;
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "gemm2: current device");
  if (rc != C3CU_OK) return rc;
  const uint32_t gen = g_split_generation.load(std::memory_order_acquire);
  std::lock_guard<std::mutex> lock(mu);
  SplitWs& entry = pool[{dev, stream}];
  if (entry.ws == nullptr) {
    rc = cuda_status(cudaMalloc(&entry.ws, kSplitWsBytes), "gemm2: split-K workspace");
    if (rc != C3CU_OK) {
      entry.ws = nullptr;
      return rc;
    }
    entry.generation = gen - 1u;  // forces the clear below
  }
  if (entry.generation != gen) {
    // cleared on the stream that will use it, so the clear precedes its next launch even on
    // a stream that does not synchronise with the legacy default stream
    rc = cuda_status(cudaMemsetAsync(entry.ws, 0, kSplitWsBytes, stream), "gemm2: clear split-K workspace");
    if (rc != C3CU_OK) return rc;
    entry.generation = gen;
  }
  *partial = static_cast<float*>(entry.ws);
  *tickets = reinterpret_cast<uint32_t*>(*partial + kSplitPartialFloats);
  *ready = *tickets + kSplitWords;
  return C3CU_OK;
}

template <bool A_MN, bool B_MN, int EPI>
int launch_pair(const void* A, int64_t lda, const void* B, int64_t ldb, const Params& p,
                cudaStream_t stream, int variant) {
  CUtensorMap ta, tb;
  int rc;
  // Per CTA: A 128 (M) x 64 (K), B 128 (N) x 64 (K); MN-major operands in 64 x 64 boxes.
  if (!A_MN)
    rc = encode_bf16_2d_sw128(&ta, A, p.M, p.K, lda, 64, gemm2::HM);
  else
    rc = encode_bf16_2d_sw128(&ta, A, p.K, p.M, lda, 64, gemm2::BK);
  if (rc != C3CU_OK) return rc;
  if (!B_MN)
    rc = encode_bf16_2d_sw128(&tb, B, p.N, p.K, ldb, 64, gemm2::HN);
  else
    rc = encode_bf16_2d_sw128(&tb, B, p.K, p.N, ldb, 64, gemm2::BK);
  if (rc != C3CU_OK) return rc;

  auto kern = gemm2::gemm2_kernel<A_MN, B_MN, EPI>;
  static std::atomic<uint64_t> smem_set{0};  // per instantiation, one bit per device
  rc = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), gemm2::SMEM_BYTES, smem_set,
                            "gemm2: set max dynamic shared memory");
  if (rc != C3CU_OK) return rc;
  const int tiles = ((p.M + gemm2::TM - 1) / gemm2::TM) * ((p.N + gemm2::TN - 1) / gemm2::TN);
  int clusters = max_pair_clusters(kern, gemm2::SMEM_BYTES, gemm2::kThreads);
  if (clusters <= 0) clusters = sm_count() / 2;
  const int cap = g_max_ctas;
  if (cap > 0 && cap / 2 < clusters) clusters = cap / 2 > 0 ? cap / 2 : 1;
  // Split-K tail (gemm2::plan_split; measured: dW with K = 2048 ran 5% slower split, hence the
  // 64-block minimum). A stream-K split of the last waves balanced the clusters exactly but ran
  // slower: the shorter pieces and their fix-ups left the tensor pipe waiting on the epilogue.
  const int k_blocks = (p.K + gemm2::BK - 1) / gemm2::BK;
  const gemm2::SplitPlan plan = gemm2::plan_split(tiles, clusters, k_blocks, variant, kSplitMax);
  Params q = p;
  q.split_wait_ns = g_split_wait_ns.load(std::memory_order_relaxed);
  q.sk_mode = plan.sk_mode;
  q.sk_first = plan.sk_first;
  clusters = plan.clusters;
  if (q.sk_mode != 0) {
    rc = split_workspace(stream, &q.partial, &q.tickets, &q.ready);
    if (rc != C3CU_OK) return rc;
  }
  return cuda_status(launch_kernel(kern, dim3(2 * clusters), dim3(gemm2::kThreads), gemm2::SMEM_BYTES, stream,
                                   ta, tb, q),
                     "gemm2: launch");
}

template <bool A_MN, bool B_MN, int EPI>
int launch(const void* A, int64_t lda, const void* B, int64_t ldb, const Params& p,
           cudaStream_t stream) {
  CUtensorMap ta, tb;
  int rc;
  // A tile: 128 (M) x 64 (K). K-major: one box {64 K, 128 rows}; MN-major: boxes {64 M, 64 K}.
  if (!A_MN)
    rc = encode_bf16_2d_sw128(&ta, A, p.M, p.K, lda, 64, gemm::BM);
  else
    rc = encode_bf16_2d_sw128(&ta, A, p.K, p.M, lda, 64, gemm::BK);
  if (rc != C3CU_OK) return rc;
  // B tile: 256 (N) x 64 (K).
  if (!B_MN)
    rc = encode_bf16_2d_sw128(&tb, B, p.N, p.K, ldb, 64, gemm::BN);
  else
    rc = encode_bf16_2d_sw128(&tb, B, p.K, p.N, ldb, 64, gemm::BK);
  if (rc != C3CU_OK) return rc;

  auto kern = gemm::gemm_kernel<A_MN, B_MN, EPI>;
  static std::atomic<uint64_t> smem_set{0};  // per instantiation, one bit per device
  rc = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), gemm::SMEM_BYTES, smem_set,
                            "gemm: set max dynamic shared memory");
  if (rc != C3CU_OK) return rc;
  const int tiles = ((p.M + gemm::BM - 1) / gemm::BM) * ((p.N + gemm::BN - 1) / gemm::BN);
  int sms = sm_count();
  const int cap = g_max_ctas;
  if (cap > 0 && cap < sms) sms = cap;
  const int grid = tiles < sms ? tiles : sms;
  return cuda_status(launch_kernel(kern, dim3(grid), dim3(gemm::kThreads), gemm::SMEM_BYTES, stream, ta, tb, p),
                     "gemm: launch");
}

int dispatch(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
             int epi, const Params& p, cudaStream_t st) {
  int variant = g_variant.load(std::memory_order_relaxed);
  {
    std::lock_guard<std::mutex> lock(g_tune_mu);
    if (!g_tune.empty()) {
      auto it = g_tune.find(TuneKey{p.M, p.N, p.K, a_mn, b_mn, epi});
      if (it != g_tune.end()) variant = it->second;
    }
  }
  const bool pair = variant != 1 && p.M > gemm2::HM;
#define C3CU_GEMM_CASE(AM, BMN, E)                                          \
  if (a_mn == AM && b_mn == BMN && epi == E)                                \
    return pair ? launch_pair<AM, BMN, E>(A, lda, B, ldb, p, st, variant)   \
                : launch<AM, BMN, E>(A, lda, B, ldb, p, st);
  C3CU_GEMM_CASE(0, 0, kEpiBiasReluMask)
  C3CU_GEMM_CASE(0, 1, kEpiBiasReluMask)
  C3CU_GEMM_CASE(0, 0, kEpiStoreBf16)
  C3CU_GEMM_CASE(0, 1, kEpiStoreBf16)
  C3CU_GEMM_CASE(1, 1, kEpiStoreF32)
  C3CU_GEMM_CASE(1, 1, kEpiStoreBf16)
  C3CU_GEMM_CASE(0, 0, kEpiStoreF32)
  C3CU_GEMM_CASE(0, 1, kEpiStoreF32)
  C3CU_GEMM_CASE(1, 0, kEpiStoreF32)
  C3CU_GEMM_CASE(0, 0, kEpiBiasStoreF32)
  C3CU_GEMM_CASE(0, 1, kEpiBiasStoreF32)
#undef C3CU_GEMM_CASE
  set_error("gemm: no kernel instantiated for a_mn=%d b_mn=%d epilogue=%d", a_mn, b_mn, epi);
  return C3CU_ERR_INVALID;
}

int check_common(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) {
    set_error("gemm: sizes out of range M=%lld N=%lld K=%lld", (long long)M, (long long)N,
              (long long)K);
    return C3CU_ERR_INVALID;
  }
  if (K == 0 && M > 0 && N > 0) {
    set_error("gemm: K == 0 is not supported (empty reduction)");
    return C3CU_ERR_INVALID;
  }
  return require_sm100();
}

}  // namespace

void gemm_invalidate_split_workspaces() { g_split_generation.fetch_add(1u, std::memory_order_acq_rel); }

int gemm_general(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                 void* out, int64_t ldo, int epi, const float* bias, uint32_t* mask, int64_t ldm,
                 int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  int rc = check_common(M, N, K);
  if (rc != C3CU_OK) return rc;
  if (M == 0 || N == 0) return C3CU_OK;
  if (!A || !B || !out) {
    set_error("gemm: null operand");
    return C3CU_ERR_INVALID;
  }
  const bool bias_epi = (epi == kEpiBiasReluMask || epi == kEpiBiasStoreF32);
  if (bias_epi && !bias) {
    set_error("gemm: epilogue %d needs a bias", epi);
    return C3CU_ERR_INVALID;
  }
  if (epi == kEpiBiasReluMask && (!mask || ldm < (N + 31) / 32)) {
    set_error("gemm: ReLU-mask epilogue needs a mask with ldm >= ceil(N/32)");
    return C3CU_ERR_INVALID;
  }
  if (ldo < N) {
    set_error("gemm: output row stride %lld < N %lld", (long long)ldo, (long long)N);
    return C3CU_ERR_INVALID;
  }
  Params p;
  p.M = static_cast<int32_t>(M);
  p.N = static_cast<int32_t>(N);
  p.K = static_cast<int32_t>(K);
  p.out = out;
  p.ldo = ldo;
  p.bias = bias;
  p.mask = mask;
  p.ldm = ldm;
  p.sk_mode = 0;
  p.sk_first = 0;
  p.partial = nullptr;
  p.tickets = nullptr;
  p.ready = nullptr;
  p.split_wait_ns = C3CU_WAIT_LIMIT_NS;
  p.ar_mc_out = nullptr;
  p.ar_mc_db = nullptr;
  p.ar_flags = nullptr;
  p.ar_mc_flags = nullptr;
  p.ar_db_count = 0;
  p.ar_rank = 0;
  p.ar_world = 1;
  p.ar_epoch = 0u;
  const int esize = (epi == kEpiStoreF32 || epi == kEpiBiasStoreF32) ? 4 : 2;
  p.vec_ok = aligned16(out) && ((ldo * esize) % 16 == 0) &&
             (!bias_epi || aligned16(bias)) ? 1 : 0;
  return dispatch(A, lda, a_mn, B, ldb, b_mn, epi, p, st);
}

}  // namespace c3cu

extern "C" {

int c3cu_set_gemm_max_ctas(int max_ctas) {
  if (max_ctas < 0) {
    c3cu::set_error("set_gemm_max_ctas: negative limit");
    return C3CU_ERR_INVALID;
  }
  c3cu::g_max_ctas = max_ctas;
  return C3CU_OK;
}

int c3cu_set_split_wait_ns(uint64_t ns) {
  c3cu::g_split_wait_ns.store(ns == 0 ? C3CU_WAIT_LIMIT_NS : ns, std::memory_order_relaxed);
  return C3CU_OK;
}

int c3cu_set_gemm_variant(int variant) {
  if (variant < 0 || variant > 2) {
    c3cu::set_error("set_gemm_variant: unknown variant %d", variant);
    return C3CU_ERR_INVALID;
  }
  c3cu::g_variant.store(variant, std::memory_order_relaxed);
  return C3CU_OK;
}

int c3cu_gemm_tune_set(int64_t M, int64_t N, int64_t K, int a_mn, int b_mn, int epilogue, int variant) {
  if (variant < 0 || variant > 2 || M < 0 || N < 0 || K < 0) {
    c3cu::set_error("gemm_tune_set: bad arguments (variant %d)", variant);
    return C3CU_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lock(c3cu::g_tune_mu);
  c3cu::g_tune[c3cu::TuneKey{M, N, K, a_mn, b_mn, epilogue}] = variant;
  return C3CU_OK;
}

int c3cu_gemm_tune_get(int64_t M, int64_t N, int64_t K, int a_mn, int b_mn, int epilogue, int* variant) {
  if (!variant) return C3CU_ERR_INVALID;
  std::lock_guard<std::mutex> lock(c3cu::g_tune_mu);
  auto it = c3cu::g_tune.find(c3cu::TuneKey{M, N, K, a_mn, b_mn, epilogue});
  if (it == c3cu::g_tune.end()) {
    c3cu::set_error("gemm_tune_get: no entry for this shape");
    return C3CU_ERR_INVALID;
  }
  *variant = it->second;
  return C3CU_OK;
}

int c3cu_gemm_tune_clear(void) {
  std::lock_guard<std::mutex> lock(c3cu::g_tune_mu);
  c3cu::g_tune.clear();
  return C3CU_OK;
}

int c3cu_gemm_bf16(const void* A, int64_t lda, int a_mn, const void* B, int64_t ldb, int b_mn,
                   void* out, int64_t ldo, int epilogue, const float* bias, uint32_t* mask,
                   int64_t ldm, int64_t M, int64_t N, int64_t K, c3cu_stream_t stream) {
  return c3cu::gemm_general(A, lda, a_mn, B, ldb, b_mn, out, ldo, epilogue, bias, mask, ldm, M,
                            N, K, static_cast<cudaStream_t>(stream));
}

int c3cu_gemm_dw_allreduce(const void* dZ, const void* X, void* dW, void* mc_dW, float* mc_db,
                           int64_t db_count, uint32_t* flags, uint32_t* mc_flags, int64_t flag_words,
                           int64_t M, int64_t N, int64_t K, int rank, int world, uint32_t epoch,
                           c3cu_stream_t stream) {
  using namespace c3cu;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // GEMM view: out dW[N][K] = dZ^T X, reduction over this rank's M rows; both operands MN-major
  int rc = check_common(N, K, M);
  if (rc != C3CU_OK) return rc;
  if (world < 1 || world > 64 || rank < 0 || rank >= world || db_count < 0) {
    set_error("gemm_dw_allreduce: bad rank %d / world %d / db_count %lld", rank, world, (long long)db_count);
    return C3CU_ERR_INVALID;
  }
  if (N == 0 || K == 0) return C3CU_OK;
  if (M == 0) {
    set_error("gemm_dw_allreduce: a rank needs at least one row (M = 0)");
    return C3CU_ERR_INVALID;
  }
  if (world == 1)  // nothing to sum: the plain dW GEMM
    return gemm_general(dZ, N, 1, X, K, 1, dW, K, kEpiStoreBf16, nullptr, nullptr, 0, N, K, M, st);
  if (!dZ || !X || !dW || !mc_dW || !flags || !mc_flags || (db_count > 0 && !mc_db)) {
    set_error("gemm_dw_allreduce: null pointer");
    return C3CU_ERR_INVALID;
  }
  if (!aligned16(dW) || !aligned16(mc_dW) || (K % 8) != 0 || (db_count % 4) != 0 ||
      (db_count > 0 && !aligned16(mc_db)) || !aligned16(flags) || !aligned16(mc_flags)) {
    set_error("gemm_dw_allreduce: dW, its multicast address, db and the flags must start on 16 bytes, "
              "K must be a multiple of 8 and db_count of 4");
    return C3CU_ERR_ALIGN;
  }
  if (N <= gemm2::HM) {
    set_error("gemm_dw_allreduce: N = %lld rows of dW; the fused kernel runs on CTA pairs and needs N > %d",
              (long long)N, gemm2::HM);
    return C3CU_ERR_INVALID;
  }
  const int64_t tiles = ((N + gemm2::TM - 1) / gemm2::TM) * ((K + gemm2::TN - 1) / gemm2::TN);
  if (flag_words < gemm2::ar::kRegion0 + gemm2::ar::kRegionsPerTile * tiles) {
    set_error("gemm_dw_allreduce: %lld flag words, %lld needed", (long long)flag_words,
              (long long)(gemm2::ar::kRegion0 + gemm2::ar::kRegionsPerTile * tiles));
    return C3CU_ERR_INVALID;
  }
  gemm::Params p;
  p.M = static_cast<int32_t>(N);
  p.N = static_cast<int32_t>(K);
  p.K = static_cast<int32_t>(M);
  p.out = dW;
  p.ldo = K;
  p.bias = nullptr;
  p.mask = nullptr;
  p.ldm = 0;
  p.vec_ok = 1;
  p.sk_mode = 0;
  p.sk_first = 0;
  p.partial = nullptr;
  p.tickets = nullptr;
  p.ready = nullptr;
  p.split_wait_ns = C3CU_WAIT_LIMIT_NS;
  p.ar_mc_out = mc_dW;
  p.ar_mc_db = mc_db;
  p.ar_flags = flags;
  p.ar_mc_flags = mc_flags;
  p.ar_db_count = static_cast<int32_t>(db_count);
  p.ar_rank = rank;
  p.ar_world = world;
  p.ar_epoch = epoch;
  return launch_pair<true, true, kEpiBf16Allreduce>(dZ, N, X, K, p, st, 0);
}

int c3cu_linear_bias_relu_fwd(const void* X, const void* W, const float* bias, void* Y,
                              uint32_t* mask, int64_t M, int64_t N, int64_t K, int w_layout,
                              c3cu_stream_t stream) {
  if (w_layout != C3CU_W_NK && w_layout != C3CU_W_KN) {
    c3cu::set_error("linear_bias_relu_fwd: unknown weight layout %d", w_layout);
    return C3CU_ERR_INVALID;
  }
  // Y[M][N] = X[M][K] * W[N][K]^T  (W K-major)  or  X[M][K] * B[K][N]  (B MN-major)
  const int64_t ldb = (w_layout == C3CU_W_NK) ? K : N;
  return c3cu::gemm_general(X, K, 0, W, ldb, w_layout == C3CU_W_KN ? 1 : 0, Y, N,
                            c3cu::kEpiBiasReluMask, bias, mask, (N + 31) / 32, M, N, K,
                            static_cast<cudaStream_t>(stream));
}

int c3cu_gemm_dx(const void* dZ, const void* W, void* dX, int64_t M, int64_t N, int64_t K,
                 int w_layout, c3cu_stream_t stream) {
  // dX[M][K] = dZ[M][N] * W[N][K]  -> GEMM (M, K, red N): A = dZ K-major, B = W stored [N][K]
  // (reduction-major = MN-major). With B[K][N]: dX = dZ * B^T, B stored [K][N] = K-major.
  if (w_layout == C3CU_W_NK)
    return c3cu::gemm_general(dZ, N, 0, W, K, 1, dX, K, c3cu::kEpiStoreBf16, nullptr, nullptr, 0,
                              M, K, N, static_cast<cudaStream_t>(stream));
  if (w_layout == C3CU_W_KN)
    return c3cu::gemm_general(dZ, N, 0, W, N, 0, dX, K, c3cu::kEpiStoreBf16, nullptr, nullptr, 0,
                              M, K, N, static_cast<cudaStream_t>(stream));
  c3cu::set_error("gemm_dx: unknown weight layout %d", w_layout);
  return C3CU_ERR_INVALID;
}

int c3cu_gemm_dw(const void* dZ, const void* X, float* dW, int64_t M, int64_t N, int64_t K,
                 int w_layout, c3cu_stream_t stream) {
  // dW[N][K] = dZ^T * X : GEMM (N, K, red M); A = dZ stored [M][N], B = X stored [M][K]
  // (both MN-major). dB[K][N] = X^T * dZ: the same with the operands swapped.
  if (w_layout == C3CU_W_NK)
    return c3cu::gemm_general(dZ, N, 1, X, K, 1, dW, K, c3cu::kEpiStoreF32, nullptr, nullptr, 0,
                              N, K, M, static_cast<cudaStream_t>(stream));
  if (w_layout == C3CU_W_KN)
    return c3cu::gemm_general(X, K, 1, dZ, N, 1, dW, N, c3cu::kEpiStoreF32, nullptr, nullptr, 0,
                              K, N, M, static_cast<cudaStream_t>(stream));
  c3cu::set_error("gemm_dw: unknown weight layout %d", w_layout);
  return C3CU_ERR_INVALID;
}

}  // extern "C"
