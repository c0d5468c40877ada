// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores (tcgen05).
//
//   D[Mg, Ng] = A[Mg, Kg] * B[Ng, Kg]^T      (fp32 accumulation in TMEM)
//
// Each operand is read by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast) in
// one of two majors, so that none of the three GEMMs of a Linear+bias+ReLU training step
// needs a physical transpose:
//   K-major  : operand stored row-major [rows][Kg]    (X and W in the forward, dZ in dX)
//   MN-major : operand stored row-major [Kg][rows]    (W in dX, dZ and X in dW)
//
// CTA = 6 warps, one CTA per SM, persistent over output tiles of 128 x 256:
//   warp 0      TMA producer (one elected lane) -> STAGES-deep smem ring (full/empty mbarriers)
//   warp 1      TMEM owner + MMA issuer (one elected lane): 4 x tcgen05.mma (K=16) per stage
//   warps 2..5  epilogue: tcgen05.ld of the accumulator quarter that warp (id % 4) may
//               access, fused epilogue, direct vector stores to global memory
// The accumulator is double-buffered in TMEM (2 x 256 fp32 columns = all 512 columns), so
// the epilogue of tile i overlaps the main loop of tile i+1.
//
// Arithmetic this kernel replaces (reference, fp32 on the host CPU): the c3.matmul
// lowering, a sequential k loop of separate fmul/fadd (src/C3/C3DialectLowering.cpp:467-610),
// followed by the FusedNode epilogue out = maxnum(T + b[j], 0) (src/C3/MLIRKernelGen.cpp:610-768).
#pragma once

#include "common.cuh"

namespace c3cu {

enum Epilogue : int {
  kEpiBiasReluMask = 0,  // out bf16 = max(acc + bias[n], 0); mask bit = (acc + bias[n] > 0)
  kEpiStoreBf16 = 1,     // out bf16 = acc
  kEpiStoreF32 = 2,      // out f32  = acc
  kEpiBiasStoreF32 = 3,  // out f32  = acc + bias[n]
  kEpiBf16Allreduce = 4, // out bf16 = acc, then summed over ranks in the NVSwitch (CTA-pair
                         // kernel only; gemm2_tcgen05.cuh, namespace ar)
};

namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int UMMA_K = 16;
constexpr int kThreads = 192;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;  // 16 KiB
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;  // 32 KiB
constexpr uint32_t STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t MN_CHUNK_BYTES = 64 * BK * 2;  // one 64-wide MN chunk of an MN-major tile
constexpr uint32_t TMEM_COLS = 512;               // two 128 x 256 fp32 accumulators
// barriers: full[S], empty[S], acc_full[2], acc_empty[2], drain; then the TMEM address slot
constexpr uint32_t BAR_BYTES = (2 * STAGES + 5) * 8 + 8;
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;  // +1 KiB alignment pad

struct Params {
  int32_t M, N, K;       // GEMM sizes (output M x N, reduction K)
  void* out;             // output base
  int64_t ldo;           // output row stride, elements
  const float* bias;     // [N] (bias epilogues)
  uint32_t* mask;        // [M][ldm] bit-packed ReLU mask (kEpiBiasReluMask)
  int64_t ldm;           // mask row stride, 32-bit words
  int32_t vec_ok;        // 1 when every 32-column chunk may use 16-byte stores
  // Work split of the CTA-pair kernel (sk_mode 0 = round robin over whole tiles; 1 = round
  // robin over the first sk_first tiles, then every remaining tile as two K halves on two
  // clusters). A tile shared by two clusters is finished by the half that takes the second
  // ticket: it adds the other half's fp32 partial (`partial`) before its epilogue.
  // `tickets` / `ready` are per-warp words that the second half returns to zero, so the
  // workspace is ready for the next launch.
  int32_t sk_mode;
  int32_t sk_first;
  float* partial;
  uint32_t* tickets;
  uint32_t* ready;
  uint64_t split_wait_ns;  // limit on the second half's wait for the first half's partial
  // kEpiBf16Allreduce: `out` is this rank's copy of a buffer bound to an NVLink multicast
  // object and `ar_mc_out` its multicast address; `ar_mc_db` the multicast address of an fp32
  // vector of `ar_db_count` elements summed alongside; `ar_flags` / `ar_mc_flags` this rank's
  // copy and the multicast address of the flag words (monotonic counters, see gemm2 ar::).
  void* ar_mc_out;
  float* ar_mc_db;
  uint32_t* ar_flags;
  uint32_t* ar_mc_flags;
  int32_t ar_db_count;
  int32_t ar_rank;
  int32_t ar_world;
  uint32_t ar_epoch;
};

template <bool A_MN, bool B_MN>
__device__ __forceinline__ void issue_stage_loads(const CUtensorMap* tma, const CUtensorMap* tmb,
                                                  uint8_t* sa, uint8_t* sb, uint64_t* bar,
                                                  int m0, int n0, int k0) {
  if constexpr (!A_MN) {
    tma_load_2d(sa, tma, bar, k0, m0);
  } else {
#pragma unroll
    for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * MN_CHUNK_BYTES, tma, bar, m0 + 64 * j, k0);
  }
  if constexpr (!B_MN) {
    tma_load_2d(sb, tmb, bar, k0, n0);
  } else {
#pragma unroll
    for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * MN_CHUNK_BYTES, tmb, bar, n0 + 64 * j, k0);
  }
}

// Bounded wait used only while draining after a fault: ignores the fault word so that the
// drain itself runs to completion (or to its own limit).
__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > C3CU_WAIT_LIMIT_NS / 4) {
      record_fault(kFaultDrain, blockIdx.x & 0xffffu);
      return false;
    }
  }
  return true;
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const Params& p, const uint32_t (&r)[32], int row,
                                               int col0) {
  if (row >= p.M) return;
  const int ncols = min(32, p.N - col0);
  const bool full_vec = p.vec_ok && ncols == 32;
  if constexpr (EPI == kEpiBiasReluMask) {
    float b[32];
    if (full_vec) {
      const float4* bp = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = __ldg(bp + j);
        b[4 * j] = v.x; b[4 * j + 1] = v.y; b[4 * j + 2] = v.z; b[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = (j < ncols) ? __ldg(p.bias + col0 + j) : 0.f;
    }
    uint32_t bits = 0u;
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float z0 = __fadd_rn(__uint_as_float(r[j]), b[j]);
      const float z1 = __fadd_rn(__uint_as_float(r[j + 1]), b[j + 1]);
      bits |= (z0 > 0.f ? 1u : 0u) << j;
      bits |= (z1 > 0.f ? 1u : 0u) << (j + 1);
      packed[j / 2] = pack_bf16x2(fmaxf(z0, 0.f), fmaxf(z1, 0.f));
    }
    if (ncols < 32) bits &= (1u << ncols) - 1u;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + col0;
    if (full_vec) {
      uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) out[j] = __ushort_as_bfloat16(static_cast<unsigned short>(packed[j >> 1] >> (16 * (j & 1))));
    }
    p.mask[(int64_t)row * p.ldm + (col0 >> 5)] = bits;
  } else if constexpr (EPI == kEpiStoreBf16) {
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2)
      packed[j / 2] = pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + col0;
    if (full_vec) {
      uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) out[j] = __ushort_as_bfloat16(static_cast<unsigned short>(packed[j >> 1] >> (16 * (j & 1))));
    }
  } else {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if constexpr (EPI == kEpiBiasStoreF32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], (j < ncols) ? __ldg(p.bias + col0 + j) : 0.f);
    }
    float* out = static_cast<float*>(p.out) + (int64_t)row * p.ldo + col0;
    if (full_vec) {
      float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) out[j] = v[j];
    }
  }
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);

  const uint32_t warp = warp_id_sync();
  const uint32_t lane = lane_id();

  const int m_tiles = (p.M + BM - 1) / BM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tma);
    tma_prefetch_desc(&tmb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel on the stream has completed (no-op without PDL)
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t armed = 0u, armed_par = 0u;  // per-stage: issued-but-unobserved, parity
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * BM;
        const int n0 = (tile % n_tiles) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, kFaultWaitEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          issue_stage_loads<A_MN, B_MN>(&tma, &tmb, sA + s * A_STAGE_BYTES, sB + s * B_STAGE_BYTES,
                                        &full[s], m0, n0, kb * BK);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok) {
        // Fault path: every copy this lane issued must land before the CTA exits.
        for (int t = 0; t < STAGES; ++t)
          if (armed & (1u << t)) drain_wait(&full[t], (armed_par >> t) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = make_idesc_bf16_f32(BM, BN, A_MN, B_MN);
      // Per UMMA_K step: K-major advances 16 elements inside the 128-byte swizzled row
      // (32 B); MN-major advances 16 K rows of 128 B (2 KiB).
      constexpr uint32_t A_KSTEP = A_MN ? UMMA_K * 128 : UMMA_K * 2;
      constexpr uint32_t B_KSTEP = B_MN ? UMMA_K * 128 : UMMA_K * 2;
      constexpr uint32_t A_LBO = A_MN ? MN_CHUNK_BYTES : 16;
      constexpr uint32_t B_LBO = B_MN ? MN_CHUNK_BYTES : 16;
      int s = 0;
      uint32_t ph = 0;
      uint32_t acc = 0, acc_ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, kFaultWaitAccEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, kFaultWaitFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t ad = make_sw128_desc(a_addr + kk * A_KSTEP, A_LBO, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + kk * B_KSTEP, B_LBO, 1024);
            umma_f16_ss(d_tmem, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // frees the smem stage once these MMAs have read it
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);  // accumulator ready for the epilogue
        acc ^= 1u;
        if (acc == 0u) acc_ph ^= 1u;
      }
      // Normal and fault exit alike: wait until every MMA this lane issued has completed.
      umma_commit(drain);
      drain_wait(drain, 0u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
    uint32_t acc = 0, acc_ph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m0 = (tile / n_tiles) * BM;
      const int n0 = (tile % n_tiles) * BN;
      if (!mbar_wait(&acc_full[acc], acc_ph, kFaultWaitAccFull)) break;
      tc_fence_after();
      const int row = m0 + static_cast<int>(q * 32 + lane);
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= p.N) break;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_wait_ld();
        epilogue_chunk<EPI>(p, r, row, col0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      acc ^= 1u;
      if (acc == 0u) acc_ph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace c3cu
