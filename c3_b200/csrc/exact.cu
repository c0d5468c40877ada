// Bit-exact fp32 kernels (CUDA cores) for the reference's fp32 arithmetic:
//   * c3cu_matmul_f32      — c3.matmul: acc = bias-or-0; for k ascending: acc = acc + a*b
//                            (separate round-to-nearest multiply and add, no FMA), then act
//                            (src/C3/C3DialectLowering.cpp:467-610)
//   * c3cu_region_fwd_f32  — MatMul+Add+ReLU region: T (as above, from 0), then
//                            out = maxnum(T + b[idx % numel(b)], 0), optional pre-activation
//                            and bit mask (src/C3/MLIRKernelGen.cpp:610-768)
//   * c3cu_sum_rows_f32_exact — SumReduce axis 0 in the reference's row order
//                            (src/C3/C3DialectLowering.cpp:382-465)
//   * c3cu_matmul_relu_bwd_f32 — the MatMul backward dA (grad @ B^T) with the next ReLU
//                            backward Mul(Gt(z, 0), .) applied to each result
//                            (src/C3/C3BackwardCapture.cpp:501-528, 681-723)
//   * c3cu_matmul_colsum_f32 — the MatMul backward dB (A^T @ grad) together with the Add
//                            backward's SumReduce of grad (src/C3/C3BackwardCapture.cpp:618-644):
//                            the column sums are one more output row whose A entries are 1, so
//                            they accumulate in the same k order, (0 + 1*g0) + 1*g1 ..., which
//                            is bit for bit SumReduce's (0 + g0) + g1 ...
// Register tiling changes which thread computes an element, never the order of the k
// reduction of that element, so these kernels reproduce the reference's results bit for
// bit (expf/tanhf of the sigmoid/tanh activations aside, which use CUDA's libm).
#include "common.cuh"
#include "host_util.h"

namespace c3cu {
namespace exact {

constexpr int TK = 32;  // k depth of one shared-memory stage
// Block tile (16 R) x (16 R): 256 threads, R x R outputs each. R = 4 for large outputs;
// R = 2 or 1 when the 64 x 64 tiles would leave most SMs idle (e.g. the cfg1 layers at
// batch 128), trading per-thread reuse for parallelism. Every output still accumulates its
// k terms in ascending order.

template <bool TA, bool TB>
__device__ __forceinline__ float load_a(const float* A, int i, int k, int M, int K) {
  if (i >= M || k >= K) return 0.f;
  return TA ? A[(int64_t)k * M + i] : A[(int64_t)i * K + k];
}

// A with one extra row of ones (row M): the column sums of B come out as output row M.
template <bool TA, bool TB>
__device__ __forceinline__ float load_a_ones(const float* A, int i, int k, int M, int K) {
  if (k >= K || i > M) return 0.f;
  if (i == M) return 1.f;
  return TA ? A[(int64_t)k * M + i] : A[(int64_t)i * K + k];
}

template <bool TA, bool TB>
__device__ __forceinline__ float load_b(const float* B, int k, int j, int K, int N) {
  if (j >= N || k >= K) return 0.f;
  return TB ? B[(int64_t)j * K + k] : B[(int64_t)k * N + j];
}

// MODE 0: out = act(bias_init + sum)     (plain c3.matmul)
// MODE 1: s = sum + b[idx % bn]; out = maxnum(s, 0); z = s; mask bits (region forward)
// MODE 2: out = (z[idx] > 0 ? 1 : 0) * sum (ReLU backward applied to dA; z is read, not written)
// MODE 3: out = sum for rows < M; row M (A's entries 1) gives the column sums of B into z
template <bool TA, bool TB, int MODE, int R>
__global__ void __launch_bounds__(256)
    sgemm_exact_kernel(const float* __restrict__ A, const float* __restrict__ B,
                       float* __restrict__ out, float* __restrict__ z, uint32_t* __restrict__ mask,
                       const float* __restrict__ bias, int64_t bias_numel, int M, int K, int N,
                       int act) {
  constexpr int TM = 16 * R, TN = 16 * R;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[R][R];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < R; ++j) {
      float init = 0.f;
      if (MODE == 0 && bias != nullptr) {
        const int col = n0 + tx * R + j;
        init = (col < N) ? bias[bias_numel == 1 ? 0 : col] : 0.f;
      }
      acc[i][j] = init;
    }
  // 256 threads move TM x TK of A and TK x TN of B per stage (LD elements each of both). The
  // next stage is fetched into registers while the current one is consumed from shared
  // memory, so the global-load latency overlaps the k loop.
  constexpr int LD = TK * 16 * R / 256;
  float ra[LD], rb[LD];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int r = 0; r < LD; ++r) {
      const int e = threadIdx.x + r * 256;
      ra[r] = MODE == 3 ? load_a_ones<TA, TB>(A, m0 + e / TK, k0 + e % TK, M, K)
                        : load_a<TA, TB>(A, m0 + e / TK, k0 + e % TK, M, K);  // A tile: [TM][TK]
      rb[r] = load_b<TA, TB>(B, k0 + e / TN, n0 + e % TN, K, N);  // B tile: [TK][TN]
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int r = 0; r < LD; ++r) {
      const int e = threadIdx.x + r * 256;
      As[e % TK][e / TK] = ra[r];
      Bs[e / TN][e % TN] = rb[r];
    }
  };
  if (K > 0) {
    fetch(0);
    stash();
  }
  for (int k0 = 0; k0 < K; k0 += TK) {
    __syncthreads();
    if (k0 + TK < K) fetch(k0 + TK);
    const int kmax = min(TK, K - k0);
    for (int kk = 0; kk < kmax; ++kk) {
      float a[R], b[R];
#pragma unroll
      for (int i = 0; i < R; ++i) a[i] = As[kk][ty * R + i];
#pragma unroll
      for (int j = 0; j < R; ++j) b[j] = Bs[kk][tx * R + j];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
    __syncthreads();
    if (k0 + TK < K) stash();
  }
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int row = m0 + ty * R + i;
    if (row > M || (row == M && MODE != 3)) continue;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int col = n0 + tx * R + j;
      if (col >= N) continue;
      const int64_t idx = (int64_t)row * N + col;
      const float t = acc[i][j];
      if (MODE == 3) {
        if (row == M)
          z[col] = t;
        else
          out[idx] = t;
      } else if (MODE == 2) {
        out[idx] = __fmul_rn(z[idx] > 0.f ? 1.f : 0.f, t);
      } else if (MODE == 0) {
        float v = t;
        if (act == 1) {
          v = fmaxf(t, 0.f);
        } else if (act == 2) {
          v = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-t)));
        } else if (act == 3) {
          v = tanhf(t);
        }
        out[idx] = v;
      } else {
        const float s = __fadd_rn(t, bias[idx % bias_numel]);
        out[idx] = fmaxf(s, 0.f);
        if (z) z[idx] = s;
        if (mask && s > 0.f) atomicOr(mask + (int64_t)row * ((N + 31) / 32) + (col >> 5), 1u << (col & 31));
      }
    }
  }
}

// One thread per column, rows ascending: the reference's accumulation order exactly.
__global__ void __launch_bounds__(256)
    sum_rows_exact_kernel(const float* __restrict__ in, float* __restrict__ out, int M, int N) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= N) return;
  float s = 0.f;
  int i = 0;
  // eight loads in flight, then added in row order (the loads do not depend on the sum)
  for (; i + 8 <= M; i += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = in[(int64_t)(i + u) * N + j];
#pragma unroll
    for (int u = 0; u < 8; ++u) s = __fadd_rn(s, v[u]);
  }
  for (; i < M; ++i) s = __fadd_rn(s, in[(int64_t)i * N + j]);
  out[j] = s;
}

template <bool TA, bool TB, int MODE, int R>
int launch_r(const float* A, const float* B, float* out, float* z, uint32_t* mask, const float* bias,
             int64_t bias_numel, int64_t M, int64_t K, int64_t N, int act, cudaStream_t st) {
  constexpr int T = 16 * R;
  const int64_t rows = MODE == 3 ? M + 1 : M;  // MODE 3: the column-sum row
  dim3 grid(static_cast<unsigned>((N + T - 1) / T), static_cast<unsigned>((rows + T - 1) / T));
  if (grid.y > 65535) {
    set_error("exact matmul: M=%lld too large", (long long)M);
    return C3CU_ERR_INVALID;
  }
  sgemm_exact_kernel<TA, TB, MODE, R><<<grid, 256, 0, st>>>(A, B, out, z, mask, bias, bias_numel,
                                                            static_cast<int>(M), static_cast<int>(K),
                                                            static_cast<int>(N), act);
  return cuda_status(cudaGetLastError(), "exact matmul: launch");
}

// Largest register tile whose grid still gives every SM at least two blocks.
template <bool TA, bool TB, int MODE>
int launch(const float* A, const float* B, float* out, float* z, uint32_t* mask, const float* bias,
           int64_t bias_numel, int64_t M, int64_t K, int64_t N, int act, cudaStream_t st) {
  const int64_t want = 2 * static_cast<int64_t>(sm_count());
  auto tiles = [&](int64_t t) { return ((M + t - 1) / t) * ((N + t - 1) / t); };
  if (tiles(64) >= want) return launch_r<TA, TB, MODE, 4>(A, B, out, z, mask, bias, bias_numel, M, K, N, act, st);
  if (tiles(32) >= want) return launch_r<TA, TB, MODE, 2>(A, B, out, z, mask, bias, bias_numel, M, K, N, act, st);
  return launch_r<TA, TB, MODE, 1>(A, B, out, z, mask, bias, bias_numel, M, K, N, act, st);
}

template <int MODE>
int dispatch(int ta, int tb, const float* A, const float* B, float* out, float* z, uint32_t* mask,
             const float* bias, int64_t bn, int64_t M, int64_t K, int64_t N, int act,
             cudaStream_t st) {
  if (!ta && !tb) return launch<false, false, MODE>(A, B, out, z, mask, bias, bn, M, K, N, act, st);
  if (!ta && tb) return launch<false, true, MODE>(A, B, out, z, mask, bias, bn, M, K, N, act, st);
  if (ta && !tb) return launch<true, false, MODE>(A, B, out, z, mask, bias, bn, M, K, N, act, st);
  return launch<true, true, MODE>(A, B, out, z, mask, bias, bn, M, K, N, act, st);
}

int check_sizes(int64_t M, int64_t K, int64_t N) {
  if (M < 0 || K < 0 || N < 0 || M > INT32_MAX || K > INT32_MAX || N > INT32_MAX) {
    set_error("exact matmul: sizes out of range");
    return C3CU_ERR_INVALID;
  }
  return require_sm100();
}

}  // namespace exact
}  // namespace c3cu

extern "C" {

int c3cu_matmul_f32(const float* A, const float* B, float* out, int64_t M, int64_t K, int64_t N,
                    int transA, int transB, const float* bias, int64_t bias_numel, int act,
                    c3cu_stream_t stream) {
  int rc = c3cu::exact::check_sizes(M, K, N);
  if (rc != C3CU_OK) return rc;
  if (M == 0 || N == 0) return C3CU_OK;
  if (!A || !B || !out || (bias && bias_numel <= 0) || act < 0 || act > 3) {
    c3cu::set_error("matmul_f32: bad arguments");
    return C3CU_ERR_INVALID;
  }
  return c3cu::exact::dispatch<0>(transA != 0, transB != 0, A, B, out, nullptr, nullptr, bias,
                                  bias_numel, M, K, N, act, static_cast<cudaStream_t>(stream));
}

int c3cu_matmul_relu_bwd_f32(const float* A, const float* B, const float* z, float* out, int64_t M, int64_t K,
                             int64_t N, int transA, int transB, c3cu_stream_t stream) {
  int rc = c3cu::exact::check_sizes(M, K, N);
  if (rc != C3CU_OK) return rc;
  if (M == 0 || N == 0) return C3CU_OK;
  if (!A || !B || !z || !out) {
    c3cu::set_error("matmul_relu_bwd_f32: null pointer");
    return C3CU_ERR_INVALID;
  }
  return c3cu::exact::dispatch<2>(transA != 0, transB != 0, A, B, out, const_cast<float*>(z), nullptr, nullptr,
                                  0, M, K, N, 0, static_cast<cudaStream_t>(stream));
}

int c3cu_matmul_colsum_f32(const float* A, const float* B, float* out, float* colsum, int64_t M, int64_t K,
                           int64_t N, int transA, int transB, c3cu_stream_t stream) {
  int rc = c3cu::exact::check_sizes(M, K, N);
  if (rc != C3CU_OK) return rc;
  if (M >= INT32_MAX) {
    c3cu::set_error("matmul_colsum_f32: M out of range");
    return C3CU_ERR_INVALID;
  }
  if (N == 0) return C3CU_OK;
  if (!out || !colsum || (K > 0 && (!B || (M > 0 && !A)))) {  // K = 0: nothing is read
    c3cu::set_error("matmul_colsum_f32: null pointer");
    return C3CU_ERR_INVALID;
  }
  return c3cu::exact::dispatch<3>(transA != 0, transB != 0, A, B, out, colsum, nullptr, nullptr, 0, M, K, N, 0,
                                  static_cast<cudaStream_t>(stream));
}

int c3cu_region_fwd_f32(const float* X, const float* B, const float* bias, int64_t bias_numel,
                        float* out, float* z, uint32_t* mask, int64_t M, int64_t K, int64_t N,
                        int transB, c3cu_stream_t stream) {
  int rc = c3cu::exact::check_sizes(M, K, N);
  if (rc != C3CU_OK) return rc;
  if (M == 0 || N == 0) return C3CU_OK;
  if (!X || !B || !out || !bias || bias_numel <= 0) {
    c3cu::set_error("region_fwd_f32: bad arguments");
    return C3CU_ERR_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mask) {
    rc = c3cu::cuda_status(
        cudaMemsetAsync(mask, 0, static_cast<size_t>(M) * static_cast<size_t>((N + 31) / 32) * 4u, st),
        "region_fwd_f32: clear mask");
    if (rc != C3CU_OK) return rc;
  }
  return c3cu::exact::dispatch<1>(0, transB != 0, X, B, out, z, mask, bias, bias_numel, M, K, N, 0,
                                  st);
}

int c3cu_sum_rows_f32_exact(const float* in, float* out, int64_t M, int64_t N,
                            c3cu_stream_t stream) {
  int rc = c3cu::exact::check_sizes(M, 1, N);
  if (rc != C3CU_OK) return rc;
  if (N == 0) return C3CU_OK;
  if (!out || (M > 0 && !in)) {
    c3cu::set_error("sum_rows_f32_exact: null pointer");
    return C3CU_ERR_INVALID;
  }
  const int grid = static_cast<int>((N + 255) / 256);
  c3cu::exact::sum_rows_exact_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      in, out, static_cast<int>(M), static_cast<int>(N));
  return c3cu::cuda_status(cudaGetLastError(), "sum_rows_f32_exact: launch");
}

}  // extern "C"
