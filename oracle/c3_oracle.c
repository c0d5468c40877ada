/*
 * c3_oracle.c — TEST INFRASTRUCTURE ONLY. A CPU restatement of the arithmetic that the
 * reference (ShengFlow/C3, a CPU MLIR/LLVM JIT) generates for the fused hot path. It is the
 * checker for the CUDA kernels and the CPU baseline timed by bench.py; nothing in the
 * product links or calls it.
 *
 * Parity status: the reference cannot be built or run (no MLIR/LLVM, no CTorch host
 * headers) and ships no tests or golden vectors, so this restatement is "parity unpinned"
 * against reference outputs. It is pinned instead to known-answer values derived by hand
 * from the reference code (tests/golden/) and cross-checked against a second, independent
 * restatement written in Python (tests/golden/make_golden.py).
 *
 * Compile with -O2 -fno-fast-math -ffp-contract=off: the JIT emits separate fmul/fadd
 * (arith.mulf / arith.addf without fastmath flags) under LLVM's default FP-op fusion
 * setting, so no multiply-add contraction happens in the reference either.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define C3O_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ GEMM (c3.matmul)
 * MatMulOpLowering (src/C3/C3DialectLowering.cpp:467-610):
 *   acc = bias ? bias[bias_numel == 1 ? 0 : j] : 0
 *   for k in 0..K-1 (ascending): acc = acc + a(i,k) * b(k,j)      (fmul then fadd)
 *   out[i*N + j] = act(acc)      act: 0 none, 1 maxnum(acc, 0), 2 1/(1+exp(-acc)), 3 tanh
 * Index maps (transpose folding, :546-562):
 *   a(i,k) = transA ? A[k*M + i] : A[i*K + k]
 *   b(k,j) = transB ? B[j*K + k] : B[k*N + j]
 * The tile loop nest (tileM x tileN) does not change any element's value: each output is
 * an independent sequential k reduction, so the oracle iterates rows directly.
 * Rows [r0, r1) only, so that large problems can be checked on sampled rows. */
static void matmul_rows(const float* A, const float* B, float* out, size_t M, size_t K,
                        size_t N, int transA, int transB, const float* bias,
                        size_t bias_numel, int act, size_t r0, size_t r1) {
  for (size_t i = r0; i < r1; ++i) {
    for (size_t j = 0; j < N; ++j) {
      float acc = 0.0f;
      if (bias) acc = bias[bias_numel == 1 ? 0 : j];
      for (size_t k = 0; k < K; ++k) {
        const float a = transA ? A[k * M + i] : A[i * K + k];
        const float b = transB ? B[j * K + k] : B[k * N + j];
        const float prod = a * b;
        acc = acc + prod;
      }
      float v = acc;
      if (act == 1) {
        v = fmaxf(acc, 0.0f);
      } else if (act == 2) {
        const float e = expf(-acc);
        const float d = 1.0f + e;
        v = 1.0f / d;
      } else if (act == 3) {
        v = tanhf(acc);
      }
      out[i * N + j] = v;
    }
  }
}

typedef struct {
  const float *A, *B, *bias;
  float* out;
  size_t M, K, N, bias_numel;
  int transA, transB, act;
  size_t r0, r1;
} mm_job;

static void* mm_worker(void* arg) {
  mm_job* j = (mm_job*)arg;
  matmul_rows(j->A, j->B, j->out, j->M, j->K, j->N, j->transA, j->transB, j->bias,
              j->bias_numel, j->act, j->r0, j->r1);
  return NULL;
}

/* Row-parallel driver: rows are split into contiguous ranges across `threads` workers;
 * every element is still computed by the serial recurrence above. */
C3O_EXPORT void c3o_matmul(const float* A, const float* B, float* out, size_t M, size_t K,
                           size_t N, int transA, int transB, const float* bias,
                           size_t bias_numel, int act, size_t r0, size_t r1, int threads) {
  if (r1 > M) r1 = M;
  if (r0 >= r1) return;
  if (threads <= 1 || r1 - r0 < 2) {
    matmul_rows(A, B, out, M, K, N, transA, transB, bias, bias_numel, act, r0, r1);
    return;
  }
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  mm_job jobs[256];
  const size_t rows = r1 - r0;
  const size_t per = (rows + (size_t)threads - 1) / (size_t)threads;
  int launched = 0;
  for (int t = 0; t < threads; ++t) {
    const size_t a = r0 + (size_t)t * per;
    if (a >= r1) break;
    const size_t b = a + per < r1 ? a + per : r1;
    mm_job j = {A, B, bias, out, M, K, N, bias_numel, transA, transB, act, a, b};
    jobs[t] = j;
    pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
    ++launched;
  }
  for (int t = 0; t < launched; ++t) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------ region forward
 * The MatMul+Add+ReLU region as the reference compiles it: Graph::fuse() turns [Add, ReLU]
 * into one FusedNode and leaves MatMul outside (src/C3/Graph.cpp:587-647), so the c3.matmul
 * gets no bias epilogue and writes T into the scratch buffer; the FusedNode loop then
 * computes out[idx] = maxnum(T[idx] + b[idx % numel(b)], 0) (src/C3/MLIRKernelGen.cpp:610-768,
 * broadcast through RemUI at :663-684). z (optional) receives T + b, the pre-activation
 * that the ReLU backward later compares with 0. Rows [r0, r1) only. */
C3O_EXPORT void c3o_region_fwd(const float* X, const float* B, const float* b, size_t b_numel,
                               float* out, float* z, size_t M, size_t K, size_t N, int transB,
                               size_t r0, size_t r1, int threads) {
  if (r1 > M) r1 = M;
  if (r0 >= r1) return;
  float* T = z ? z : out;
  c3o_matmul(X, B, T, M, K, N, 0, transB, NULL, 0, 0, r0, r1, threads);
  for (size_t i = r0; i < r1; ++i) {
    for (size_t j = 0; j < N; ++j) {
      const size_t idx = i * N + j;
      const float s = T[idx] + b[idx % b_numel];
      if (z) z[idx] = s;
      out[idx] = fmaxf(s, 0.0f);
    }
  }
}

/* ------------------------------------------------------------------ ReLU backward
 * buildReLUBackwardGraph: Mul(Gt(x, 0), grad) (src/C3/C3BackwardCapture.cpp:501-528);
 * Gt is CmpF OGT selecting 1.0f / 0.0f, so NaN compares false (src/C3/MLIRKernelGen.cpp:173-211). */
C3O_EXPORT void c3o_relu_bwd(const float* grad, const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float g = (x[i] > 0.0f) ? 1.0f : 0.0f;
    out[i] = g * grad[i];
  }
}

/* The same with the pre-activation given as the packed bit mask the forward kernel emits:
 * bit (j & 31) of word mask[i*ldm + j/32] is 1 iff z[i][j] > 0. */
C3O_EXPORT void c3o_relu_bwd_mask(const float* grad, const uint32_t* mask, size_t ldm,
                                  float* out, size_t M, size_t N) {
  for (size_t i = 0; i < M; ++i)
    for (size_t j = 0; j < N; ++j) {
      const float g = ((mask[i * ldm + j / 32] >> (j & 31)) & 1u) ? 1.0f : 0.0f;
      out[i * N + j] = g * grad[i * N + j];
    }
}

/* ------------------------------------------------------------------ SumReduce axis 0
 * SumReduceOpLowering (src/C3/C3DialectLowering.cpp:382-465): out[j] = 0, then for rows
 * i ascending out[j] = out[j] + in[i*N + j]. Axis 1: the same along each row. */
C3O_EXPORT void c3o_sum_reduce(const float* in, float* out, size_t M, size_t N, int axis) {
  if (axis == 0) {
    for (size_t j = 0; j < N; ++j) {
      out[j] = 0.0f;
      for (size_t i = 0; i < M; ++i) out[j] = out[j] + in[i * N + j];
    }
  } else {
    for (size_t i = 0; i < M; ++i) {
      out[i] = 0.0f;
      for (size_t j = 0; j < N; ++j) out[i] = out[i] + in[i * N + j];
    }
  }
}

/* ------------------------------------------------------------------ elementwise chains
 * relu((A + B) * C - A) / (1 + exp(-B)) exactly as the reference graph evaluates it:
 * Neg, Exp and Add(Const 1, .) are separate nodes that materialise d = 1 + expf(-B); the
 * FusedNode [Add, Mul, Sub, ReLU, Div] then runs per element (src/C3/MLIRKernelGen.cpp:394-605
 * for the unbroadcast, vectorised form: plain fdiv). Up to `threads` workers over contiguous
 * ranges, mirroring the <=8-thread slicing of large elementwise kernels
 * (src/C3/C3Engine.cpp:164-211). */
typedef struct {
  const float *A, *B, *C;
  float* out;
  size_t lo, hi;
} ew_job;

static void ew_cfg4_range(const float* A, const float* B, const float* C, float* out, size_t lo,
                          size_t hi) {
  for (size_t i = lo; i < hi; ++i) {
    const float nb = -B[i];
    const float e = expf(nb);
    const float d = 1.0f + e;
    const float s = A[i] + B[i];
    const float m = s * C[i];
    const float t = m - A[i];
    const float r = fmaxf(t, 0.0f);
    out[i] = r / d;
  }
}

static void* ew_worker(void* arg) {
  ew_job* j = (ew_job*)arg;
  ew_cfg4_range(j->A, j->B, j->C, j->out, j->lo, j->hi);
  return NULL;
}

C3O_EXPORT void c3o_ew_cfg4(const float* A, const float* B, const float* C, float* out, size_t n,
                            int threads) {
  if (threads <= 1 || n < 2) {
    ew_cfg4_range(A, B, C, out, 0, n);
    return;
  }
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  ew_job jobs[256];
  const size_t per = (n + (size_t)threads - 1) / (size_t)threads;
  int launched = 0;
  for (int t = 0; t < threads; ++t) {
    const size_t lo = (size_t)t * per;
    if (lo >= n) break;
    const size_t hi = lo + per < n ? lo + per : n;
    ew_job j = {A, B, C, out, lo, hi};
    jobs[t] = j;
    pthread_create(&tid[t], NULL, ew_worker, &jobs[t]);
    ++launched;
  }
  for (int t = 0; t < launched; ++t) pthread_join(tid[t], NULL);
}

/* General chain with the same register-machine encoding as c3cu_ew_program: 4-byte
 * instructions {op, dst, src0, src1}; registers 0..n_inputs-1 are loaded from
 * inputs[i][idx % numels[i]]. Operation semantics follow the scalar FusedNode loop
 * (src/C3/MLIRKernelGen.cpp:660-767) and the Linalg generic bodies
 * (src/C3/LinalgFusedGen.cpp:211-362). Opcode values match include/c3cu.h. */
C3O_EXPORT void c3o_ew_program(const float* const* inputs, const int64_t* numels, int n_inputs,
                               const uint8_t* code, int n_instr, const float* constants,
                               int out_reg, float* out, int64_t n) {
  for (int64_t idx = 0; idx < n; ++idx) {
    float reg[16];
    memset(reg, 0, sizeof(reg));
    for (int i = 0; i < n_inputs; ++i) reg[i] = inputs[i][idx % numels[i]];
    for (int k = 0; k < n_instr; ++k) {
      const int op = code[4 * k], dst = code[4 * k + 1], s0 = code[4 * k + 2], s1 = code[4 * k + 3];
      const float a = reg[s0], b = reg[s1];
      float v;
      switch (op) {
        case 1: v = a + b; break;
        case 2: v = a - b; break;
        case 3: v = a * b; break;
        case 4: v = a / b; break;
        case 5: v = (b == 0.0f) ? NAN : a / b; break;
        case 6: v = -a; break;
        case 7: v = fmaxf(a, 0.0f); break;
        case 8: v = expf(a); break;
        case 9: v = logf(a); break;
        case 10: { const float e = expf(-a); const float d = 1.0f + e; v = 1.0f / d; } break;
        case 11: v = tanhf(a); break;
        case 12: {
          const float ep = expf(a), en = expf(-a);
          const float num = ep - en, den = ep + en;
          v = num / den;
        } break;
        case 13: v = (a > b) ? 1.0f : 0.0f; break;
        case 14: v = constants[s0]; break;
        case 15: v = a; break;
        default: v = NAN; break;
      }
      reg[dst] = v;
    }
    out[idx] = reg[out_reg];
  }
}

/* ------------------------------------------------------------------ attention (no reference)
 * The reference has no attention kernel. Textbook causal softmax attention in fp32 for the
 * rows [q0, q1) of one (batch, head): O = softmax(scale * Q K^T + causal mask) V and
 * LSE = m + log(sum exp(s - m)) in natural log. q, k, v: [S][D] row-major. */
C3O_EXPORT void c3o_attention_rows(const float* q, const float* k, const float* v, float* o,
                                   float* lse, size_t S, size_t D, float scale, int causal,
                                   size_t q0, size_t q1, float* scratch /* [S] */) {
  for (size_t i = q0; i < q1 && i < S; ++i) {
    const size_t jmax = causal ? i + 1 : S;
    float m = -INFINITY;
    for (size_t j = 0; j < jmax; ++j) {
      double dot = 0.0;
      for (size_t d = 0; d < D; ++d) dot += (double)q[i * D + d] * (double)k[j * D + d];
      scratch[j] = (float)(dot * (double)scale);
      if (scratch[j] > m) m = scratch[j];
    }
    double l = 0.0;
    for (size_t j = 0; j < jmax; ++j) {
      scratch[j] = (float)exp((double)scratch[j] - (double)m);
      l += scratch[j];
    }
    for (size_t d = 0; d < D; ++d) {
      double acc = 0.0;
      for (size_t j = 0; j < jmax; ++j) acc += (double)scratch[j] * (double)v[j * D + d];
      o[i * D + d] = (float)(acc / l);
    }
    if (lse) lse[i] = (float)((double)m + log(l));
  }
}

/* ------------------------------------------------------------------ training step (cfg1)
 * The reference trains its MLP with the host framework's loss and optimizer, which are not
 * part of the reference sources (CTorch): these are the textbook definitions, in the order
 * the CUDA kernels use (parity unpinned).
 * Softmax cross-entropy, mean over B rows:
 *   m = max_c z[i][c]; s = sum_c expf(z[i][c] - m) (c ascending); lse = m + logf(s)
 *   loss = (sum_i (lse_i - z[i][y_i])) / B   (i ascending; the product with 1/B)
 *   dz[i][c] = (expf(z[i][c] - lse_i) - (c == y_i)) * (1 / B)
 * A label outside [0, C) makes that row's loss (so the total) and its dz row NaN. */
C3O_EXPORT void c3o_softmax_ce(const float* z, const int32_t* y, float* loss, float* dz, size_t B, size_t C) {
  const float invB = 1.f / (float)B;
  float total = 0.f;
  for (size_t i = 0; i < B; ++i) {
    const float* zr = z + i * C;
    float* dr = dz ? dz + i * C : NULL;
    const int32_t label = y[i];
    float li;
    if (label < 0 || (size_t)label >= C) {
      li = NAN;
      if (dr)
        for (size_t c = 0; c < C; ++c) dr[c] = NAN;
    } else {
      float m = zr[0];
      for (size_t c = 1; c < C; ++c) m = fmaxf(m, zr[c]);
      float s = 0.f;
      for (size_t c = 0; c < C; ++c) s = s + expf(zr[c] - m);
      const float lse = m + logf(s);
      li = lse - zr[label];
      if (dr)
        for (size_t c = 0; c < C; ++c) {
          const float pc = expf(zr[c] - lse);
          dr[c] = (pc - ((int32_t)c == label ? 1.f : 0.f)) * invB;
        }
    }
    total = total + li;
  }
  *loss = total * invB;
}

/* SGD: p[i] = p[i] - lr * g[i] (multiply, then subtract). */
C3O_EXPORT void c3o_sgd(float* p, const float* g, size_t n, float lr) {
  for (size_t i = 0; i < n; ++i) p[i] = p[i] - lr * g[i];
}

/* ------------------------------------------------------------------ fused backward chains
 * The gradient graphs the reference builds per unary node (src/C3/C3BackwardCapture.cpp:
 * 501-617 ReLU/Sigmoid/Tanh, 725-743 Neg, 823-872 Exp/Log), chained from the most
 * downstream node (k = 0) upstream as the fused sequence kernel does (:1133-1210); each
 * graph node is one IEEE fp32 operation (the fused graphs compile without secondary fusion,
 * :1236-1246). ops: 1 ReLU, 2 Sigmoid, 3 Tanh, 4 Neg, 5 Exp, 6 Log. outs[k] = the gradient
 * node k passes upstream. */
C3O_EXPORT void c3o_backward_chain(const int* ops, int n_nodes, const float* grad, const float* const* xs,
                                   float* const* outs, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float g = grad[i];
    for (int k = 0; k < n_nodes; ++k) {
      const float x = xs[k] ? xs[k][i] : 0.f;
      float r;
      switch (ops[k]) {
        case 1: r = (x > 0.f ? 1.f : 0.f) * g; break;
        case 2: {
          const float e = expf(-x);
          const float s = 1.f / (1.f + e);
          r = g * (s * (1.f - s));
          break;
        }
        case 3: {
          const float ep = expf(x), en = expf(-x);
          const float t = (ep - en) / (ep + en);
          r = g * (1.f - t * t);
          break;
        }
        case 4: r = -g; break;
        case 5: r = expf(x) * g; break;
        case 6: r = g / x; break;
        default: r = NAN; break;
      }
      outs[k][i] = r;
      g = r;
    }
  }
}
