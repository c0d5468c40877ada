// Loss and optimizer kernels of the cfg1 MLP training step (include/c3cu.h):
//   * c3cu_softmax_ce_f32 — softmax cross-entropy over C classes, mean over B rows, and its
//                           gradient with respect to the logits, in one kernel
//   * c3cu_sgd_f32        — plain SGD, p <- p - lr * g, over up to C3CU_SGD_MAX_TENSORS tensors
//                           in one launch
// The reference trains its MLP with the host framework's own loss and optimizer (CTorch,
// outside the C3 hot path, not part of the reference sources), so these follow the textbook
// definitions; fp32 throughout, each operation rounded separately (no contraction), in the
// order the CPU oracle uses.
#include "common.cuh"
#include "host_util.h"

C3CU_FAULT_ACCESSORS(train)

namespace c3cu {
namespace train {

constexpr int kCeThreads = 512;
constexpr int kCeSeqRows = 8192;  // up to this many rows the loss is summed rows-ascending

// One CTA. Row i (thread-strided):
//   m = max_c z[i][c];  s = sum_c exp(z[i][c] - m) (c ascending);  lse = m + log(s)
//   loss_i = lse - z[i][y_i];  dz[i][c] = (exp(z[i][c] - lse) - (c == y_i)) * (1 / B)
// loss = (sum_i loss_i) / B. A label outside [0, C) makes loss_i (and the loss) NaN and its
// row of dz NaN.
__global__ void __launch_bounds__(kCeThreads)
    softmax_ce_kernel(const float* __restrict__ z, const int32_t* __restrict__ y, float* __restrict__ loss,
                      float* __restrict__ dz, int B, int C) {
  __shared__ float row_loss[kCeSeqRows];
  __shared__ float part[kCeThreads];
  const float invB = 1.f / static_cast<float>(B);
  float acc = 0.f;  // used when B > kCeSeqRows
  for (int i = threadIdx.x; i < B; i += blockDim.x) {
    const float* zr = z + static_cast<int64_t>(i) * C;
    float* dr = dz ? dz + static_cast<int64_t>(i) * C : nullptr;
    const int label = y[i];
    float li;
    if (label < 0 || label >= C) {
      li = __int_as_float(0x7fc00000);
      if (dr)
        for (int c = 0; c < C; ++c) dr[c] = li;
    } else {
      float m = zr[0];
      for (int c = 1; c < C; ++c) m = fmaxf(m, zr[c]);
      float s = 0.f;
      for (int c = 0; c < C; ++c) s = __fadd_rn(s, expf(__fsub_rn(zr[c], m)));
      const float lse = __fadd_rn(m, logf(s));
      li = __fsub_rn(lse, zr[label]);
      if (dr)
        for (int c = 0; c < C; ++c) {
          const float pc = expf(__fsub_rn(zr[c], lse));
          dr[c] = __fmul_rn(__fsub_rn(pc, c == label ? 1.f : 0.f), invB);
        }
    }
    if (B <= kCeSeqRows)
      row_loss[i] = li;
    else
      acc = __fadd_rn(acc, li);
  }
  if (B <= kCeSeqRows) {
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < B; ++i) t = __fadd_rn(t, row_loss[i]);
      *loss = __fmul_rn(t, invB);
    }
  } else {
    // fixed-shape tree over the per-thread partial sums (deterministic, not rows-ascending)
    part[threadIdx.x] = acc;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if (static_cast<int>(threadIdx.x) < w) part[threadIdx.x] = __fadd_rn(part[threadIdx.x], part[threadIdx.x + w]);
      __syncthreads();
    }
    if (threadIdx.x == 0) *loss = __fmul_rn(part[0], invB);
  }
}

struct SgdArgs {
  float* p[C3CU_SGD_MAX_TENSORS];
  const float* g[C3CU_SGD_MAX_TENSORS];
  int64_t end[C3CU_SGD_MAX_TENSORS];  // exclusive prefix sums of the element counts
  int count;
  float lr;
};

__global__ void __launch_bounds__(256) sgd_kernel(const SgdArgs a) {
  const int64_t total = a.end[a.count - 1];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < total; k += stride) {
    int t = 0;
    while (k >= a.end[t]) ++t;
    const int64_t i = k - (t == 0 ? 0 : a.end[t - 1]);
    a.p[t][i] = __fsub_rn(a.p[t][i], __fmul_rn(a.lr, a.g[t][i]));
  }
}

}  // namespace train
}  // namespace c3cu

extern "C" int c3cu_softmax_ce_f32(const float* logits, const int32_t* labels, float* loss, float* dlogits,
                                   int64_t B, int64_t C, c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (B <= 0 || C <= 0 || B > INT32_MAX || C > INT32_MAX || !logits || !labels || !loss) {
    set_error("softmax_ce_f32: bad arguments (B %lld, C %lld)", (long long)B, (long long)C);
    return C3CU_ERR_INVALID;
  }
  train::softmax_ce_kernel<<<1, train::kCeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, labels, loss, dlogits, static_cast<int>(B), static_cast<int>(C));
  return cuda_status(cudaGetLastError(), "softmax_ce_f32: launch");
}

extern "C" int c3cu_sgd_f32(float* const* params, const float* const* grads, const int64_t* numels, int count,
                            float lr, c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (count < 1 || count > C3CU_SGD_MAX_TENSORS || !params || !grads || !numels) {
    set_error("sgd_f32: 1 to %d tensors expected, got %d", C3CU_SGD_MAX_TENSORS, count);
    return C3CU_ERR_INVALID;
  }
  train::SgdArgs a{};
  int64_t total = 0;
  for (int t = 0; t < count; ++t) {
    if (numels[t] < 0 || (numels[t] > 0 && (!params[t] || !grads[t]))) {
      set_error("sgd_f32: tensor %d: bad pointer or size", t);
      return C3CU_ERR_INVALID;
    }
    a.p[t] = params[t];
    a.g[t] = grads[t];
    total += numels[t];
    a.end[t] = total;
  }
  a.count = count;
  a.lr = lr;
  if (total == 0) return C3CU_OK;
  const int64_t blocks = (total + 255) / 256;
  const int grid = static_cast<int>(blocks < 4 * sm_count() ? blocks : 4 * sm_count());
  train::sgd_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cuda_status(cudaGetLastError(), "sgd_f32: launch");
}
