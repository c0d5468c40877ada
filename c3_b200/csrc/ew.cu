// HBM-bound kernels of the C3 hot path (include/c3cu.h):
//   * c3cu_relu_mask_db   — ReLU backward dZ = float(mask) * dY fused with the Add-backward
//                           column sum db = sum_rows dZ (deterministic two-level reduction)
//   * c3cu_sum_rows_f32   — SumReduce axis 0 over an fp32 matrix
//   * c3cu_ew_chain_cfg4  — relu((A + B) * C - A) / (1 + exp(-B)) in one pass
//   * c3cu_ew_program     — general single-pass elementwise chain (register-machine program)
//
// All of them stream with 128-bit loads/stores, coalesced across each warp, and size the
// grid as a multiple of the SM count. Floating-point operations are written with the
// explicit round-to-nearest intrinsics (__fadd_rn, __fmul_rn, ...) so that the compiler
// cannot contract them into FMAs: the reference evaluates each node as a separate fp32
// operation (src/C3/MLIRKernelGen.cpp:394-768), and the kernels keep that order.
#include <mutex>
#include <vector>

#include "common.cuh"
#include "host_util.h"

C3CU_FAULT_ACCESSORS(ew)

namespace c3cu {
namespace ew {

constexpr int kColsPerWarp = 256;   // 32 lanes x 8 columns
constexpr int kWarps = 8;
constexpr int kRowsPerBlock = 512;  // rows one block reduces before the cross-block pass
#ifndef C3CU_COLSUM_PREFETCH
#define C3CU_COLSUM_PREFETCH 1
#endif
constexpr bool kColsumPrefetch = C3CU_COLSUM_PREFETCH != 0;

// L2 prefetch of `bytes` (a multiple of 16) from a 16-byte-aligned global address; no data is
// returned and no register is held.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------ column sums
// One block covers a strip of 256 columns and up to 512 rows. Each thread owns 8 adjacent
// columns; warps stride over rows. The block writes its 256 partial sums to
// `partials[row_block][col]`; the last block of a strip to finish (atomic ticket) adds the
// partials of that strip in row-block order, so the result does not depend on scheduling.
//
// MASKED: input bf16 dY with a bit-packed mask; also writes dZ = float(bit) * dY as bf16
//         (reference: Mul(Gt(x, 0), grad), src/C3/C3BackwardCapture.cpp:501-528, where
//         Gt yields 1.0f / 0.0f, src/C3/MLIRKernelGen.cpp:173-211).
// !MASKED: input fp32, sum only (SumReduce axis 0, src/C3/C3DialectLowering.cpp:382-465).
// Loads the 8 values a thread owns in row r (bf16 dY with its mask bits, or fp32).
template <bool MASKED>
__device__ __forceinline__ void colsum_load(const void* __restrict__ in, const uint32_t* __restrict__ mask,
                                            int r, int col, int N, int ldm, bool vec, uint32_t (&raw)[8],
                                            uint32_t& bits) {
  if constexpr (MASKED) {
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(in) + (int64_t)r * N + col;
    if (vec) {
      const uint4 q = __ldcs(reinterpret_cast<const uint4*>(src));
      raw[0] = q.x; raw[1] = q.y; raw[2] = q.z; raw[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = (col + 2 * j < N) ? __bfloat16_as_ushort(src[2 * j]) : 0u;
        const uint32_t hi = (col + 2 * j + 1 < N) ? __bfloat16_as_ushort(src[2 * j + 1]) : 0u;
        raw[j] = lo | (hi << 16);
      }
    }
    bits = __ldg(mask + (int64_t)r * ldm + (col >> 5)) >> (col & 31);
  } else {
    const float* src = static_cast<const float*>(in) + (int64_t)r * N + col;
    if (vec) {
      const uint4 a = __ldcs(reinterpret_cast<const uint4*>(src));
      const uint4 b = __ldcs(reinterpret_cast<const uint4*>(src) + 1);
      raw[0] = a.x; raw[1] = a.y; raw[2] = a.z; raw[3] = a.w;
      raw[4] = b.x; raw[5] = b.y; raw[6] = b.z; raw[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) raw[j] = (col + j < N) ? __float_as_uint(src[j]) : 0u;
    }
    bits = 0u;
  }
}

// Processes row r from the loaded values: writes dZ (MASKED) and accumulates.
template <bool MASKED>
__device__ __forceinline__ void colsum_consume(__nv_bfloat16* __restrict__ dz, int r, int col, int N, bool vec,
                                               const uint32_t (&raw)[8], uint32_t bits, float (&acc)[8]) {
  float v[8];
  if constexpr (MASKED) {
    uint32_t outw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g0 = __uint_as_float(raw[j] << 16);
      const float g1 = __uint_as_float(raw[j] & 0xffff0000u);
      v[2 * j] = __fmul_rn((bits >> (2 * j)) & 1u ? 1.f : 0.f, g0);
      v[2 * j + 1] = __fmul_rn((bits >> (2 * j + 1)) & 1u ? 1.f : 0.f, g1);
      // v is exactly g or a signed zero, so the bf16 repacking is exact.
      outw[j] = (__float_as_uint(v[2 * j]) >> 16) | (__float_as_uint(v[2 * j + 1]) & 0xffff0000u);
    }
    __nv_bfloat16* dst = dz + (int64_t)r * N + col;
    if (vec) {
      __stcs(reinterpret_cast<uint4*>(dst), make_uint4(outw[0], outw[1], outw[2], outw[3]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (col + j < N) dst[j] = __ushort_as_bfloat16(static_cast<unsigned short>(outw[j >> 1] >> (16 * (j & 1))));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(raw[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], v[j]);
}

// One block covers a strip of 256 columns and `rows_per_block` rows. Each thread owns 8
// adjacent columns; warps stride over rows, four rows at a time with all loads issued
// before any is consumed (memory-level parallelism). The block writes its 256 partial
// sums to `partials[row_block][col]`; the last block of a strip to finish (atomic ticket)
// adds the partials of that strip in row-block order, so the result does not depend on
// scheduling.
//
// MASKED: input bf16 dY with a bit-packed mask; also writes dZ = float(bit) * dY as bf16
//         (reference: Mul(Gt(x, 0), grad), src/C3/C3BackwardCapture.cpp:501-528, where
//         Gt yields 1.0f / 0.0f, src/C3/MLIRKernelGen.cpp:173-211).
// !MASKED: input fp32, sum only (SumReduce axis 0, src/C3/C3DialectLowering.cpp:382-465).
template <bool MASKED>
__global__ void __launch_bounds__(kWarps * 32)
    colsum_kernel(const void* __restrict__ in, const uint32_t* __restrict__ mask,
                  __nv_bfloat16* __restrict__ dz, float* __restrict__ out, int M, int N,
                  int ldm, int rows_per_block, float* __restrict__ partials,
                  unsigned int* __restrict__ tickets, int vec_ok) {
  __shared__ float red[kWarps][kColsPerWarp];
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int strip = blockIdx.x;
  const int rb = blockIdx.y;
  const int col = strip * kColsPerWarp + lane * 8;
  const int row0 = rb * rows_per_block;
  const int row1 = min(M, row0 + rows_per_block);

  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  pdl_wait();  // the previous kernel on the stream has completed (no-op without PDL)
  pdl_launch_dependents();

  if (col < N) {
    const bool vec = vec_ok && (col + 8 <= N);
    int r = row0 + warp;
    // Rows of the next batch are prefetched into L2 (one bulk prefetch of the warp's row segment,
    // issued by lane 0) while this batch is consumed: twice the DRAM requests in flight per
    // warp without more registers. Only whole 16-byte-aligned segments of valid rows.
    const int seg_cols = min(kColsPerWarp, N - strip * kColsPerWarp);
    const uint32_t seg_bytes = static_cast<uint32_t>(seg_cols) * (MASKED ? 2u : 4u);
    const bool prefetch = kColsumPrefetch && vec_ok && lane == 0 && (seg_bytes & 15u) == 0u;
    const char* seg0 = static_cast<const char*>(in) +
                       static_cast<int64_t>(strip) * kColsPerWarp * (MASKED ? 2 : 4);
    const int64_t row_bytes = static_cast<int64_t>(N) * (MASKED ? 2 : 4);
    for (; r + 3 * kWarps < row1; r += 4 * kWarps) {
      uint32_t raw[4][8], bits[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) colsum_load<MASKED>(in, mask, r + u * kWarps, col, N, ldm, vec, raw[u], bits[u]);
      if (prefetch) {
#pragma unroll
        for (int u = 4; u < 8; ++u) {
          const int rn = r + u * kWarps;
          if (rn < row1) prefetch_l2_bulk(seg0 + rn * row_bytes, seg_bytes);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) colsum_consume<MASKED>(dz, r + u * kWarps, col, N, vec, raw[u], bits[u], acc);
    }
    for (; r < row1; r += kWarps) {
      uint32_t raw[8], bits;
      colsum_load<MASKED>(in, mask, r, col, N, ldm, vec, raw, bits);
      colsum_consume<MASKED>(dz, r, col, N, vec, raw, bits, acc);
    }
  }

#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = acc[j];
  __syncthreads();
  // thread t adds column t of the strip over the 8 warps, in warp order
  const int t = threadIdx.x;
  const int c = strip * kColsPerWarp + t;
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s = __fadd_rn(s, red[w][t]);
  if (c < N) partials[(int64_t)rb * N + c] = s;
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const unsigned int ticket = atomicAdd(&tickets[strip], 1u);
    is_last = (ticket == gridDim.y - 1);
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
    if (c < N) {
      float tot = 0.f;
      for (int b = 0; b < static_cast<int>(gridDim.y); ++b)
        tot = __fadd_rn(tot, __ldcg(partials + (int64_t)b * N + c));
      out[c] = tot;
    }
    if (t == 0) tickets[strip] = 0u;  // re-arm for the next launch on this workspace
  }
}

// Rows per block: enough blocks to fill the SMs several times over (at least 4 per SM),
// between 64 and 512 rows, a multiple of the 8 warps x 4-row batches.
int64_t colsum_rows_per_block(int64_t M, int64_t N) {
  const int64_t strips = (N + kColsPerWarp - 1) / kColsPerWarp;
  const int64_t target_blocks = 4 * 148;
  int64_t rows = (M * strips + target_blocks - 1) / target_blocks;
  rows = (rows + 31) / 32 * 32;
  if (rows < 64) rows = 64;
  if (rows > kRowsPerBlock) rows = kRowsPerBlock;
  return rows;
}

size_t colsum_workspace(int64_t M, int64_t N) {
  const int64_t rbs = (M + colsum_rows_per_block(M, N) - 1) / colsum_rows_per_block(M, N);
  const int64_t strips = (N + kColsPerWarp - 1) / kColsPerWarp;
  const size_t partial_bytes = static_cast<size_t>(rbs > 0 ? rbs : 1) * static_cast<size_t>(N) * 4u;
  const size_t ticket_bytes = static_cast<size_t>(strips > 0 ? strips : 1) * 4u;
  return ((partial_bytes + 255u) & ~static_cast<size_t>(255u)) + ticket_bytes;
}

// Strip tickets owned by the library, one array per (device, stream), zeroed once when it
// is created. Every launch leaves its tickets at zero (the last block of a strip re-arms
// its ticket), so launches on the stream need no clearing pass of their own; launches on
// different streams never share an array.
constexpr int64_t kPoolStrips = 1 << 16;

int ticket_pool(cudaStream_t st, unsigned int** out) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, cudaStream_t>, void*>> pool;
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "column sum: current device");
  if (rc != C3CU_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : pool)
    if (e.first.first == dev && e.first.second == st) {
      *out = static_cast<unsigned int*>(e.second);
      return C3CU_OK;
    }
  void* p = nullptr;
  rc = cuda_status(cudaMalloc(&p, kPoolStrips * 4), "column sum: ticket array");
  if (rc != C3CU_OK) return rc;
  // cleared on the stream that will use it (ordered before its first launch on any stream kind)
  rc = cuda_status(cudaMemsetAsync(p, 0, kPoolStrips * 4, st), "column sum: clear ticket array");
  if (rc != C3CU_OK) {
    cudaFree(p);
    return rc;
  }
  pool.push_back({{dev, st}, p});
  *out = static_cast<unsigned int*>(p);
  return C3CU_OK;
}

// `pooled`: take the strip tickets from the library's per-stream array (no clearing pass);
// otherwise they live in the caller's workspace and are cleared before the kernel.
template <bool MASKED>
int launch_colsum(const void* in, const uint32_t* mask, void* dz, float* out, int64_t M, int64_t N,
                  void* ws, size_t ws_bytes, cudaStream_t st, bool pooled = true) {
  if (M < 0 || N < 0 || M > INT32_MAX || N > INT32_MAX) {
    set_error("column sum: sizes out of range");
    return C3CU_ERR_INVALID;
  }
  if (N == 0) return C3CU_OK;
  if (!out || (M > 0 && !in) || (MASKED && M > 0 && (!mask || !dz))) {
    set_error("column sum: null pointer");
    return C3CU_ERR_INVALID;
  }
  if (M == 0) {
    // Empty reduction: every column sums to +0.
    return cuda_status(cudaMemsetAsync(out, 0, static_cast<size_t>(N) * 4u, st), "column sum: zero");
  }
  const size_t need = colsum_workspace(M, N);
  if (!ws || ws_bytes < need) {
    set_error("column sum: workspace of %zu bytes needed, %zu given", need, ws ? ws_bytes : 0);
    return C3CU_ERR_WORKSPACE;
  }
  const int64_t rpb = colsum_rows_per_block(M, N);
  const int64_t rbs = (M + rpb - 1) / rpb;
  const int64_t strips = (N + kColsPerWarp - 1) / kColsPerWarp;
  if (rbs > 65535) {
    set_error("column sum: M=%lld exceeds %lld rows", (long long)M, (long long)65535 * rpb);
    return C3CU_ERR_INVALID;
  }
  float* partials = static_cast<float*>(ws);
  const size_t partial_bytes = static_cast<size_t>(rbs) * static_cast<size_t>(N) * 4u;
  unsigned int* tickets = reinterpret_cast<unsigned int*>(
      static_cast<uint8_t*>(ws) + ((partial_bytes + 255u) & ~static_cast<size_t>(255u)));
  int rc = C3CU_OK;
  if (pooled && strips <= kPoolStrips) {
    rc = ticket_pool(st, &tickets);
  } else {
    rc = cuda_status(cudaMemsetAsync(tickets, 0, static_cast<size_t>(strips) * 4u, st),
                     "column sum: reset tickets");
  }
  if (rc != C3CU_OK) return rc;
  const int esize = MASKED ? 2 : 4;
  const int vec_ok = aligned16(in) && (!MASKED || aligned16(dz)) && ((N * esize) % 16 == 0);
  const int ldm = static_cast<int>((N + 31) / 32);
  dim3 grid(static_cast<unsigned>(strips), static_cast<unsigned>(rbs));
  return cuda_status(launch_kernel(colsum_kernel<MASKED>, grid, dim3(kWarps * 32), 0, st, in, mask,
                                   static_cast<__nv_bfloat16*>(dz), out, static_cast<int>(M),
                                   static_cast<int>(N), ldm, static_cast<int>(rpb), partials, tickets, vec_ok),
                     "column sum: launch");
}

// ------------------------------------------------------------------ cfg4 chain
__device__ __forceinline__ float chain_cfg4(float a, float b, float c) {
  // Graph order of relu((A + B) * C - A) / (1 + exp(-B)): FusedNode [Add, Mul, Sub, ReLU, Div]
  // with the divisor 1 + exp(-B) computed by the separate Neg, Exp, Add nodes.
  const float s = __fadd_rn(a, b);
  const float m = __fmul_rn(s, c);
  const float t = __fsub_rn(m, a);
  const float r = fmaxf(t, 0.f);
  const float d = __fadd_rn(1.f, expf(-b));
  return __fdiv_rn(r, d);
}

__device__ __forceinline__ float4 chain_cfg4_v(float4 a, float4 b, float4 c) {
  return make_float4(chain_cfg4(a.x, b.x, c.x), chain_cfg4(a.y, b.y, c.y), chain_cfg4(a.z, b.z, c.z),
                     chain_cfg4(a.w, b.w, c.w));
}

// Grid-stride over float4s; each iteration issues 4 float4 loads per input (12 x 16 B in
// flight per thread) before computing, which keeps HBM busy at the measured copy bandwidth.
constexpr int kCfg4Unroll = 4;

__global__ void __launch_bounds__(256)
    chain_cfg4_kernel(const float* __restrict__ A, const float* __restrict__ B,
                      const float* __restrict__ C, float* __restrict__ out, int64_t n, int vec_ok) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t T = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec_ok) {
    const int64_t n4 = n >> 2;
    const float4* A4 = reinterpret_cast<const float4*>(A);
    const float4* B4 = reinterpret_cast<const float4*>(B);
    const float4* C4 = reinterpret_cast<const float4*>(C);
    float4* O4 = reinterpret_cast<float4*>(out);
    int64_t i = tid;
    for (; i + (kCfg4Unroll - 1) * T < n4; i += kCfg4Unroll * T) {
      float4 a[kCfg4Unroll], b[kCfg4Unroll], c[kCfg4Unroll];
#pragma unroll
      for (int u = 0; u < kCfg4Unroll; ++u) {
        a[u] = __ldcs(A4 + i + u * T);
        b[u] = __ldcs(B4 + i + u * T);
        c[u] = __ldcs(C4 + i + u * T);
      }
#pragma unroll
      for (int u = 0; u < kCfg4Unroll; ++u) __stcs(O4 + i + u * T, chain_cfg4_v(a[u], b[u], c[u]));
    }
    for (; i < n4; i += T) __stcs(O4 + i, chain_cfg4_v(__ldcs(A4 + i), __ldcs(B4 + i), __ldcs(C4 + i)));
    for (int64_t k = (n4 << 2) + tid; k < n; k += T) out[k] = chain_cfg4(A[k], B[k], C[k]);
  } else {
    for (int64_t k = tid; k < n; k += T) out[k] = chain_cfg4(A[k], B[k], C[k]);
  }
}

// ------------------------------------------------------------------ general chain
struct Program {
  const float* in[C3CU_EW_MAX_INPUTS];
  int64_t numel[C3CU_EW_MAX_INPUTS];
  uint32_t code[C3CU_EW_MAX_INSTR];  // {op, dst, src0, src1} packed little-endian
  float consts[16];
  float* out[C3CU_EW_MAX_OUTPUTS];
  int out_reg[C3CU_EW_MAX_OUTPUTS];
  int n_inputs;
  int n_instr;
  int n_out;
};

__device__ __forceinline__ float ew_apply(uint32_t op, float a, float b, float cst) {
  switch (op) {
    case C3CU_EW_ADD: return __fadd_rn(a, b);
    case C3CU_EW_SUB: return __fsub_rn(a, b);
    case C3CU_EW_MUL: return __fmul_rn(a, b);
    case C3CU_EW_DIV: return __fdiv_rn(a, b);
    case C3CU_EW_DIV_NANZ: return b == 0.f ? __int_as_float(0x7fc00000) : __fdiv_rn(a, b);
    case C3CU_EW_NEG: return -a;
    case C3CU_EW_RELU: return fmaxf(a, 0.f);
    case C3CU_EW_EXP: return expf(a);
    case C3CU_EW_LOG: return logf(a);
    case C3CU_EW_SIGMOID: return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-a)));
    case C3CU_EW_TANH: return tanhf(a);
    case C3CU_EW_TANH_EXP: {
      const float ep = expf(a), en = expf(-a);
      return __fdiv_rn(__fsub_rn(ep, en), __fadd_rn(ep, en));
    }
    case C3CU_EW_GT: return a > b ? 1.f : 0.f;
    case C3CU_EW_CONST: return cst;
    case C3CU_EW_MOV: return a;
    default: return __int_as_float(0x7fc00000);
  }
}

// Registers live in a per-thread array; each thread evaluates the program on 4 adjacent
// elements so that every decoded instruction is amortised over a 128-bit vector.
__global__ void __launch_bounds__(256) program_kernel(const Program prog, int64_t n) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = tid * 4; base < n; base += nthreads * 4) {
    float reg[16][4];
    const bool full = base + 4 <= n;
    for (int i = 0; i < prog.n_inputs; ++i) {
      const float* p = prog.in[i];
      const int64_t ne = prog.numel[i];
      if (ne == n && full && ((reinterpret_cast<uintptr_t>(p + base) & 15u) == 0u)) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(p + base));
        reg[i][0] = v.x; reg[i][1] = v.y; reg[i][2] = v.z; reg[i][3] = v.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t idx = base + e;
          reg[i][e] = (idx < n) ? __ldg(p + (ne == n ? idx : idx % ne)) : 0.f;
        }
      }
    }
    for (int k = 0; k < prog.n_instr; ++k) {
      const uint32_t w = prog.code[k];
      const uint32_t op = w & 0xffu, dst = (w >> 8) & 0xfu, s0 = (w >> 16) & 0xfu, s1 = (w >> 24) & 0xfu;
      const float cst = prog.consts[s0];
#pragma unroll
      for (int e = 0; e < 4; ++e) reg[dst][e] = ew_apply(op, reg[s0][e], reg[s1][e], cst);
    }
    for (int j = 0; j < prog.n_out; ++j) {
      const int o = prog.out_reg[j];
      float* out = prog.out[j];
      if (full && ((reinterpret_cast<uintptr_t>(out + base) & 15u) == 0u)) {
        __stcs(reinterpret_cast<float4*>(out + base), make_float4(reg[o][0], reg[o][1], reg[o][2], reg[o][3]));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (base + e < n) out[base + e] = reg[o][e];
      }
    }
  }
}

__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ in,
                                                          __nv_bfloat16* __restrict__ out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __float2bfloat16_rn(in[i]);
}

__global__ void __launch_bounds__(256) bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ in,
                                                          float* __restrict__ out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = __bfloat162float(in[i]);
}

int grid_for(int64_t work_items, int threads, int blocks_per_sm = 8) {
  const int64_t sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t want = (work_items + threads - 1) / threads;
  const int64_t cap = sms * blocks_per_sm;
  int64_t g = want < cap ? want : cap;
  return static_cast<int>(g > 0 ? g : 1);
}

}  // namespace ew
}  // namespace c3cu

// ------------------------------------------------------------------ allocation-free scratch
// Scratch of c3cu_relu_mask_db_noalloc: a fixed array in device global memory that the
// library owns. Every GPU that loads the library holds C3CU_NOALLOC_SCRATCH_BYTES of it
// until the process exits. Host code must not pass `g_noalloc_scratch` itself to a kernel
// (on the host that name is a stand-in, not a device address): the address is looked up
// once per device (and CUDA context) with cudaGetSymbolAddress and cached.
static __device__ __align__(256) uint8_t g_noalloc_scratch[C3CU_NOALLOC_SCRATCH_BYTES];

namespace c3cu {
namespace ew {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
// The address is cached per device together with the CUDA context it was looked up in: after
// a cudaDeviceReset the runtime makes a new primary context, the library's module is loaded
// again and the array may sit elsewhere, so a different current context forces a new lookup.
struct NoallocSlot {
  CUcontext ctx;
  void* addr;
};
NoallocSlot g_noalloc[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

CUcontext current_context() {
  CUcontext ctx = nullptr;
  CtxGetCurrentFn f = ctx_get_current_fn();
  if (f == nullptr || f(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of the scratch array on the current device. The first call on a device (and
// the first after that device's context was replaced) performs the lookup, so it should
// happen before any stream capture. Without a current context the lookup runs every call.
int noalloc_scratch(void** out) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), "relu_mask_db_noalloc: cudaGetDevice");
  if (rc != C3CU_OK) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("relu_mask_db_noalloc: device ordinal %d out of range", dev);
    return C3CU_ERR_UNSUPPORTED;
  }
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc[dev];
  if (slot.addr == nullptr || ctx == nullptr || slot.ctx != ctx) {
    void* p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                     "relu_mask_db_noalloc: cudaGetSymbolAddress of the scratch array");
    if (rc != C3CU_OK) return rc;
    // the lookup made the runtime's context current if none was
    slot.ctx = ctx != nullptr ? ctx : current_context();
    slot.addr = p;
  }
  *out = slot.addr;
  return C3CU_OK;
}
}  // namespace
}  // namespace ew
}  // namespace c3cu

extern "C" {

size_t c3cu_relu_mask_db_workspace(int64_t M, int64_t N) { return c3cu::ew::colsum_workspace(M, N); }

int c3cu_relu_mask_db(const void* dY, const uint32_t* mask, void* dZ, float* db, int64_t M,
                      int64_t N, void* workspace, size_t workspace_bytes, c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  return c3cu::ew::launch_colsum<true>(dY, mask, dZ, db, M, N, workspace, workspace_bytes,
                                       static_cast<cudaStream_t>(stream));
}

int c3cu_relu_mask_db_noalloc(const void* dY, const uint32_t* mask, void* dZ, float* db,
                              int64_t M, int64_t N, c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  if (M < 0 || N < 0) {
    c3cu::set_error("relu_mask_db_noalloc: negative size");
    return C3CU_ERR_INVALID;
  }
  const size_t need = c3cu::ew::colsum_workspace(M, N);
  if (need > C3CU_NOALLOC_SCRATCH_BYTES) {
    c3cu::set_error("relu_mask_db_noalloc: M=%lld N=%lld needs %zu bytes of scratch, more than the "
                    "%d-byte built-in array; use c3cu_relu_mask_db with a caller workspace",
                    (long long)M, (long long)N, need, C3CU_NOALLOC_SCRATCH_BYTES);
    return C3CU_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  rc = c3cu::ew::noalloc_scratch(&scratch);
  if (rc != C3CU_OK) return rc;
  // launch_colsum clears the ticket counters in the scratch before the kernel; the partial
  // sums are fully written before they are read, so stale contents from earlier calls are harmless.
  return c3cu::ew::launch_colsum<true>(dY, mask, dZ, db, M, N, scratch, C3CU_NOALLOC_SCRATCH_BYTES,
                                       static_cast<cudaStream_t>(stream), /*pooled=*/false);
}

size_t c3cu_sum_rows_f32_workspace(int64_t M, int64_t N) { return c3cu::ew::colsum_workspace(M, N); }

int c3cu_sum_rows_f32(const float* in, float* out, int64_t M, int64_t N, void* workspace,
                      size_t workspace_bytes, c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  return c3cu::ew::launch_colsum<false>(in, nullptr, nullptr, out, M, N, workspace,
                                        workspace_bytes, static_cast<cudaStream_t>(stream));
}

int c3cu_ew_chain_cfg4(const float* A, const float* B, const float* C, float* out, int64_t n,
                       c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  if (n < 0) {
    c3cu::set_error("ew_chain_cfg4: negative size");
    return C3CU_ERR_INVALID;
  }
  if (n == 0) return C3CU_OK;
  if (!A || !B || !C || !out) {
    c3cu::set_error("ew_chain_cfg4: null pointer");
    return C3CU_ERR_INVALID;
  }
  const int vec_ok = c3cu::aligned16(A) && c3cu::aligned16(B) && c3cu::aligned16(C) &&
                     c3cu::aligned16(out);
  const int grid = c3cu::ew::grid_for((n + 15) / 16, 256, 16);
  c3cu::ew::chain_cfg4_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(A, B, C, out, n,
                                                                                   vec_ok);
  return c3cu::cuda_status(cudaGetLastError(), "ew_chain_cfg4: launch");
}

int c3cu_convert(const void* in, int in_dtype, void* out, int out_dtype, int64_t n,
                 c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  if (n < 0 || (n > 0 && (!in || !out))) {
    c3cu::set_error("convert: bad arguments");
    return C3CU_ERR_INVALID;
  }
  if (n == 0) return C3CU_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = c3cu::ew::grid_for(n, 256);
  if (in_dtype == out_dtype) {
    const size_t bytes = static_cast<size_t>(n) * (in_dtype == C3CU_DTYPE_BF16 ? 2u : 4u);
    return c3cu::cuda_status(cudaMemcpyAsync(out, in, bytes, cudaMemcpyDeviceToDevice, st), "convert: copy");
  }
  if (in_dtype == C3CU_DTYPE_F32 && out_dtype == C3CU_DTYPE_BF16)
    c3cu::ew::f32_to_bf16_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(in),
                                                       static_cast<__nv_bfloat16*>(out), n);
  else if (in_dtype == C3CU_DTYPE_BF16 && out_dtype == C3CU_DTYPE_F32)
    c3cu::ew::bf16_to_f32_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(in),
                                                       static_cast<float*>(out), n);
  else {
    c3cu::set_error("convert: unsupported dtypes %d -> %d", in_dtype, out_dtype);
    return C3CU_ERR_INVALID;
  }
  return c3cu::cuda_status(cudaGetLastError(), "convert: launch");
}

int c3cu_ew_program_multi(const float* const* inputs, const int64_t* numels, int n_inputs,
                          const uint8_t* code, int n_instr, const float* constants, int n_constants,
                          const int* out_regs, float* const* outs, int n_out, int64_t n,
                          c3cu_stream_t stream) {
  int rc = c3cu::require_sm100();
  if (rc != C3CU_OK) return rc;
  if (n < 0 || n_inputs < 0 || n_inputs > C3CU_EW_MAX_INPUTS || n_instr < 0 ||
      n_instr > C3CU_EW_MAX_INSTR || n_constants < 0 || n_constants > 16 || n_out < 1 ||
      n_out > C3CU_EW_MAX_OUTPUTS || !out_regs || !outs) {
    c3cu::set_error("ew_program: bad program shape (inputs %d, instructions %d, constants %d, outputs %d)",
                    n_inputs, n_instr, n_constants, n_out);
    return C3CU_ERR_INVALID;
  }
  if (n == 0) return C3CU_OK;
  if ((n_inputs > 0 && (!inputs || !numels)) || (n_instr > 0 && !code)) {
    c3cu::set_error("ew_program: null pointer");
    return C3CU_ERR_INVALID;
  }
  c3cu::ew::Program prog{};
  prog.n_inputs = n_inputs;
  prog.n_instr = n_instr;
  prog.n_out = n_out;
  for (int j = 0; j < n_out; ++j) {
    if (out_regs[j] < 0 || out_regs[j] > 15 || !outs[j]) {
      c3cu::set_error("ew_program: output %d: bad register %d or null pointer", j, out_regs[j]);
      return C3CU_ERR_INVALID;
    }
    prog.out_reg[j] = out_regs[j];
    prog.out[j] = outs[j];
  }
  for (int i = 0; i < n_inputs; ++i) {
    if (!inputs[i] || numels[i] <= 0) {
      c3cu::set_error("ew_program: input %d is null or empty", i);
      return C3CU_ERR_INVALID;
    }
    if (numels[i] != n && n % numels[i] != 0 && numels[i] > n) {
      c3cu::set_error("ew_program: input %d has %lld elements, output %lld", i,
                      (long long)numels[i], (long long)n);
      return C3CU_ERR_INVALID;
    }
    prog.in[i] = inputs[i];
    prog.numel[i] = numels[i];
  }
  for (int k = 0; k < n_instr; ++k) {
    const uint8_t op = code[4 * k], dst = code[4 * k + 1], s0 = code[4 * k + 2], s1 = code[4 * k + 3];
    if (op < C3CU_EW_ADD || op > C3CU_EW_MOV || dst > 15 || s0 > 15 || s1 > 15 ||
        (op == C3CU_EW_CONST && s0 >= n_constants)) {
      c3cu::set_error("ew_program: bad instruction %d {%u,%u,%u,%u}", k, op, dst, s0, s1);
      return C3CU_ERR_INVALID;
    }
    prog.code[k] = static_cast<uint32_t>(op) | (static_cast<uint32_t>(dst) << 8) |
                   (static_cast<uint32_t>(s0) << 16) | (static_cast<uint32_t>(s1) << 24);
  }
  for (int c = 0; c < n_constants; ++c) prog.consts[c] = constants[c];
  const int grid = c3cu::ew::grid_for((n + 3) / 4, 256);
  c3cu::ew::program_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(prog, n);
  return c3cu::cuda_status(cudaGetLastError(), "ew_program: launch");
}

int c3cu_ew_program(const float* const* inputs, const int64_t* numels, int n_inputs,
                    const uint8_t* code, int n_instr, const float* constants, int n_constants,
                    int out_reg, float* out, int64_t n, c3cu_stream_t stream) {
  float* outs[1] = {out};
  return c3cu_ew_program_multi(inputs, numels, n_inputs, code, n_instr, constants, n_constants, &out_reg,
                               outs, 1, n, stream);
}

// Fused backward of a chain of unary elementwise nodes in one pass. Each node's gradient is
// the graph the reference builds for it (src/C3/C3BackwardCapture.cpp:501-617, 725-743,
// 823-872), one IEEE operation per graph node (the fused backward graphs are compiled without
// secondary fusion, :1236-1246, so Div is a plain division):
//   ReLU     Mul(Gt(x, 0), g)
//   Sigmoid  s = Div(1, Add(1, Exp(Neg(x)))); Mul(g, Mul(s, Sub(1, s)))
//   Tanh     t = Div(Sub(Exp(x), Exp(Neg(x))), Add(Exp(x), Exp(Neg(x)))); Mul(g, Sub(1, Mul(t, t)))
//   Neg      Neg(g)
//   Exp      Mul(Exp(x), g)
//   Log      Div(g, x)
// Registers: 0 = incoming gradient, 1..N = the nodes' forward inputs, then each node's
// output gradient, then temporaries (constant table: 0 -> 0.0, 1 -> 1.0).
int c3cu_ew_backward_chain(const int* node_ops, int n_nodes, const float* grad, const float* const* xs,
                           float* const* outs, int64_t n, c3cu_stream_t stream) {
  if (!node_ops || n_nodes < 1 || n_nodes > C3CU_BW_MAX_CHAIN || !grad || !outs) {
    c3cu::set_error("ew_backward_chain: 1 to %d nodes expected, got %d", C3CU_BW_MAX_CHAIN, n_nodes);
    return C3CU_ERR_INVALID;
  }
  std::vector<uint8_t> code;
  auto emit = [&](int op, int dst, int s0, int s1) {
    code.push_back(static_cast<uint8_t>(op));
    code.push_back(static_cast<uint8_t>(dst));
    code.push_back(static_cast<uint8_t>(s0));
    code.push_back(static_cast<uint8_t>(s1));
  };
  const float* inputs[C3CU_EW_MAX_INPUTS] = {grad};
  int64_t numels[C3CU_EW_MAX_INPUTS] = {n};
  int n_inputs = 1 + n_nodes;
  for (int k = 0; k < n_nodes; ++k) {
    const int op = node_ops[k];
    if (op < C3CU_BW_RELU || op > C3CU_BW_LOG) {
      c3cu::set_error("ew_backward_chain: node %d has unknown type %d", k, op);
      return C3CU_ERR_INVALID;
    }
    const float* x = xs ? xs[k] : nullptr;
    if (op != C3CU_BW_NEG && !x) {
      c3cu::set_error("ew_backward_chain: node %d needs its forward input", k);
      return C3CU_ERR_INVALID;
    }
    inputs[1 + k] = x ? x : grad;  // Neg reads no forward input; any valid pointer will do
    numels[1 + k] = n;
  }
  const int t0 = 1 + 2 * n_nodes, t1 = t0 + 1, t2 = t0 + 2;  // temporaries (<= 11, 12, 13)
  int g = 0;
  int out_regs[C3CU_EW_MAX_OUTPUTS];
  for (int k = 0; k < n_nodes; ++k) {
    const int x = 1 + k, o = 1 + n_nodes + k;
    switch (node_ops[k]) {
      case C3CU_BW_RELU:
        emit(C3CU_EW_CONST, t0, 0, 0);
        emit(C3CU_EW_GT, t0, x, t0);
        emit(C3CU_EW_MUL, o, t0, g);
        break;
      case C3CU_BW_SIGMOID:
        emit(C3CU_EW_NEG, t0, x, 0);
        emit(C3CU_EW_EXP, t0, t0, 0);
        emit(C3CU_EW_CONST, t1, 1, 0);
        emit(C3CU_EW_ADD, t0, t1, t0);
        emit(C3CU_EW_DIV, t0, t1, t0);  // s
        emit(C3CU_EW_SUB, t2, t1, t0);
        emit(C3CU_EW_MUL, t0, t0, t2);
        emit(C3CU_EW_MUL, o, g, t0);
        break;
      case C3CU_BW_TANH:
        emit(C3CU_EW_EXP, t0, x, 0);
        emit(C3CU_EW_NEG, t1, x, 0);
        emit(C3CU_EW_EXP, t1, t1, 0);
        emit(C3CU_EW_SUB, t2, t0, t1);
        emit(C3CU_EW_ADD, t0, t0, t1);
        emit(C3CU_EW_DIV, t0, t2, t0);  // t
        emit(C3CU_EW_MUL, t0, t0, t0);
        emit(C3CU_EW_CONST, t1, 1, 0);
        emit(C3CU_EW_SUB, t0, t1, t0);
        emit(C3CU_EW_MUL, o, g, t0);
        break;
      case C3CU_BW_NEG:
        emit(C3CU_EW_NEG, o, g, 0);
        break;
      case C3CU_BW_EXP:
        emit(C3CU_EW_EXP, t0, x, 0);
        emit(C3CU_EW_MUL, o, t0, g);
        break;
      case C3CU_BW_LOG:
        emit(C3CU_EW_DIV, o, g, x);
        break;
    }
    out_regs[k] = o;
    g = o;
  }
  const float consts[2] = {0.f, 1.f};
  return c3cu_ew_program_multi(inputs, numels, n_inputs, code.data(), static_cast<int>(code.size() / 4), consts,
                               2, out_regs, outs, n_nodes, n, stream);
}

}  // extern "C"
