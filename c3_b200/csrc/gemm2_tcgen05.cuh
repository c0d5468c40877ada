// CTA-pair variant of the persistent tcgen05 GEMM (cta_group::2), same operands, majors and
// epilogues as gemm_tcgen05.cuh:
//
//   D[Mg, Ng] = A[Mg, Kg] * B[Ng, Kg]^T      (fp32 accumulation in TMEM)
//
// A cluster of two CTAs (one TPC) computes 256 x 256 output tiles. Each CTA loads its own
// 128 rows of A and its own 128 of the tile's 256 B rows (N), so a CTA moves 32 KiB per
// 64-deep K block instead of 48 KiB for the single-CTA 128 x 256 tile: one third less
// L2 -> shared-memory traffic per output element. The even CTA ("leader") issues one
// 256 x 256 x 16 tcgen05.mma per K step, which reads both CTAs' shared memory and writes
// each CTA's half of the accumulator rows into that CTA's TMEM.
//
// Which tiles (and K ranges) a cluster computes comes from gemm2_schedule.h (work_item), the
// same header the launcher's split plan and the host-side coverage test use.
//
// Roles per CTA (10 warps, one CTA per SM):
//   warp 0      TMA producer. Both CTAs load their halves; every copy signals the leader's
//               `full` barrier (the leader arms it with the bytes of both halves).
//   warp 1      TMEM owner (pair allocation); in the leader also the MMA issuer. Each
//               stage is released in both CTAs by one multicast tcgen05.commit.
//   warps 2..9  epilogue on this CTA's 128 accumulator rows, two warps per TMEM lane
//               quarter (warp w reads lanes 32 * (w % 4) ...), each on half of the 256
//               columns; they release an accumulator by arriving on the leader's
//               `acc_empty` barrier (16 arrivals: both CTAs).
// Loads use no cluster multicast: every CTA reads its own operands from global memory.
#pragma once

#include "gemm2_schedule.h"
#include "gemm_tcgen05.cuh"
#include "multimem.cuh"

namespace c3cu {
namespace gemm2 {

constexpr int TM = 256;          // output tile rows per pair (128 per CTA)
constexpr int TN = 256;          // output tile columns per pair
constexpr int HM = TM / 2;       // A rows per CTA
constexpr int HN = TN / 2;       // B rows (output columns) loaded per CTA
constexpr int BK = 64;
constexpr int STAGES = 7;
constexpr int UMMA_K = 16;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t A_STAGE_BYTES = HM * BK * 2;  // 16 KiB
constexpr uint32_t B_STAGE_BYTES = HN * BK * 2;  // 16 KiB
constexpr uint32_t STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t MN_CHUNK_BYTES = 64 * BK * 2;
constexpr uint32_t TMEM_COLS = 512;  // two accumulators of 128 lanes x 256 fp32 columns
constexpr uint32_t BAR_BYTES = (2 * STAGES + 5) * 8 + 8;
constexpr uint32_t SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
constexpr uint16_t kPairMask = 0x3;

template <bool A_MN, bool B_MN>
__device__ __forceinline__ void issue_half_loads(const CUtensorMap* tma, const CUtensorMap* tmb,
                                                 uint8_t* sa, uint8_t* sb, uint32_t bar_leader,
                                                 int a_row0, int b_row0, int k0) {
  if constexpr (!A_MN) {
    tma_load_2d_pair(sa, tma, bar_leader, k0, a_row0);
  } else {
#pragma unroll
    for (int j = 0; j < HM / 64; ++j)
      tma_load_2d_pair(sa + j * MN_CHUNK_BYTES, tma, bar_leader, a_row0 + 64 * j, k0);
  }
  if constexpr (!B_MN) {
    tma_load_2d_pair(sb, tmb, bar_leader, k0, b_row0);
  } else {
#pragma unroll
    for (int j = 0; j < HN / 64; ++j)
      tma_load_2d_pair(sb + j * MN_CHUNK_BYTES, tmb, bar_leader, b_row0 + 64 * j, k0);
  }
}

// Fault path of a CTA that cannot observe the barrier its copies signal (the peer's copies
// complete on the leader's barrier): give copies already in flight time to land before the
// CTA's shared memory is released. A copy of a few KiB lands within microseconds.
__device__ __forceinline__ void settle_inflight_copies() {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < 200000ull) {
  }
}

// One unit of a cluster's work: an output tile and the K blocks [kb0, kb1) to accumulate.
// split >= 0 marks a tile that two clusters share as two K halves (the index of its fp32
// partial slot); the two halves meet through a ticket in the epilogue.
// Bounded acquire-wait for a split partner's "partial published" word.
__device__ __forceinline__ bool wait_ready(const uint32_t* flag, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t v;
  while (true) {
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v != 0u) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      record_fault(kFaultWaitPeer, blockIdx.x & 0xffffu);
      return false;
    }
  }
}

// ---------------------------------------------------------------- fused all-reduce epilogue
// kEpiBf16Allreduce: the data-parallel dW GEMM sums its output over the ranks while it runs.
// Every rank computes the same tiles in the same order (its own partial dW, from its rows of
// the batch). An epilogue warp owns a region of 32 rows x 128 columns of a tile; after storing
// its bf16 partial there it adds 1 to the region's counter in every rank's copy
// (multimem.red.release). Once the counter shows all ranks, rank r's warp reduces slice r of
// the region through the NVSwitch (multimem.ld_reduce with fp32 accumulation) and writes the
// sum into every rank's copy (multimem.st). The reduction of a region is deferred by one tile,
// so the ranks' progress on it has a tile's time to line up. db (fp32, already summed locally
// by the pre-pass) is reduced the same way by the first CTA before its first tile.
// Completion: each CTA takes a local ticket after its reductions; the last CTA of a rank adds 1
// to the completion counter of every rank and waits until all ranks have arrived, so when the
// kernel ends on a rank, dW and db hold the sums everywhere. Only that CTA waits at the end,
// so CTAs of one grid never wait for one another. Counters only grow: launch e (the same on
// every rank) waits for world * (e + 1). Every wait is bounded.
namespace ar {
constexpr int kDbFlag = 0;      // db: ranks whose pre-pass output is ready
constexpr int kDoneFlag = 1;    // ranks whose reductions are all issued
constexpr int kTicket = 2;      // this rank's CTAs that finished (local; zero between launches)
constexpr int kRegion0 = 4;     // then 16 counters per output tile
constexpr int kRegionsPerTile = 16;
constexpr uint64_t kWaitNs = C3CU_WAIT_LIMIT_NS / 2;

__device__ __forceinline__ uint32_t target(const gemm::Params& p) {
  return static_cast<uint32_t>(p.ar_world) * (p.ar_epoch + 1u);
}

// After the warp's stores to its region: make them visible system-wide, then count the region.
__device__ __forceinline__ void signal_region(const gemm::Params& p, uint32_t region, uint32_t lane) {
  __syncwarp();
  if (lane == 0) {
    mm::fence_sys();
    mm::red_release_add(p.ar_mc_flags + kRegion0 + region, 1u);
  }
  __syncwarp();
}

// This rank's slice of the region (rows row0.., columns col0..col0+127) once every rank stored
// it: 512 16-byte vectors, slice r of world, up to 8 switch round trips in flight per lane.
__device__ __forceinline__ void reduce_region(const gemm::Params& p, uint32_t region, int row0, int col0,
                                              uint32_t lane) {
  uint32_t ok = 1u;
  if (lane == 0) ok = mm::wait_counter(p.ar_flags + kRegion0 + region, target(p), kWaitNs, region) ? 1u : 0u;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return;
  constexpr int kVecs = 32 * 16;
  const int per = (kVecs + p.ar_world - 1) / p.ar_world;
  const int v0 = p.ar_rank * per;
  const int v1 = min(kVecs, v0 + per);
  uint8_t* base = static_cast<uint8_t*>(p.ar_mc_out);
  for (int vb = v0; vb < v1; vb += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int vi = vb + u * 32 + static_cast<int>(lane);
      const int r = row0 + vi / 16;
      const int c = col0 + (vi % 16) * 8;
      if (vi < v1 && r < p.M && c < p.N) mm::ld_reduce_bf16x8(base + ((int64_t)r * p.ldo + c) * 2, v[u]);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int vi = vb + u * 32 + static_cast<int>(lane);
      const int r = row0 + vi / 16;
      const int c = col0 + (vi % 16) * 8;
      if (vi < v1 && r < p.M && c < p.N) mm::st_bf16x8(base + ((int64_t)r * p.ldo + c) * 2, v[u]);
    }
  }
}

// db: the first CTA's eight epilogue warps (thread t = 32 * warp + lane, 256 threads) sum this
// rank's slice of db over the ranks, before their first tile.
__device__ __forceinline__ void reduce_db(const gemm::Params& p, uint32_t ew, uint32_t lane) {
  const int t = static_cast<int>(ew * 32u + lane);
  if (t == 0) {
    mm::fence_sys();
    mm::red_release_add(p.ar_mc_flags + kDbFlag, 1u);
  }
  uint32_t ok = 1u;
  if (lane == 0) ok = mm::wait_counter(p.ar_flags + kDbFlag, target(p), kWaitNs, 0xfffeu) ? 1u : 0u;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok || p.ar_db_count <= 0) return;
  const int nvec = p.ar_db_count / 4;
  const int per = (nvec + p.ar_world - 1) / p.ar_world;
  const int v0 = p.ar_rank * per;
  const int v1 = min(nvec, v0 + per);
  for (int v = v0 + t; v < v1; v += 256) {
    float4 x;
    mm::ld_reduce_f32x4(p.ar_mc_db + 4 * v, x);
    mm::st_f32x4(p.ar_mc_db + 4 * v, x);
  }
}

// End of the epilogue of one CTA (all eight epilogue warps call it).
__device__ __forceinline__ void finish(const gemm::Params& p, uint32_t ew, uint32_t lane) {
  asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight epilogue warps' reductions are issued
  if (ew == 0 && lane == 0) {
    mm::fence_sys();
    const uint32_t t = atomicAdd(p.ar_flags + kTicket, 1u);
    if (t == gridDim.x - 1u) {
      p.ar_flags[kTicket] = 0u;  // every CTA of this launch has taken its ticket
      mm::fence_sys();
      mm::red_release_add(p.ar_mc_flags + kDoneFlag, 1u);
      mm::wait_counter(p.ar_flags + kDoneFlag, target(p), kWaitNs, 0xffffu);
    }
  }
  __syncwarp();
}
}  // namespace ar

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                 const gemm::Params p) {
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
  const uint32_t rank = cluster_ctarank();  // 0 = leader
  const bool leader = rank == 0u;
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int num_clusters = static_cast<int>(gridDim.x >> 1);

  const int m_tiles = (p.M + TM - 1) / TM;
  const int n_tiles = (p.N + TN - 1) / TN;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tma);
    tma_prefetch_desc(&tmb);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM of the pair allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel on the stream has completed (no-op without PDL)
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t armed = 0u, armed_par = 0u;
      bool ok = true;
      Item it;
      for (int i = 0; ok && work_item(i, cluster, num_clusters, num_tiles, p.sk_mode, p.sk_first, k_blocks, it);
           ++i) {
        const int m0 = (it.tile / n_tiles) * TM;
        const int n0 = (it.tile % n_tiles) * TN;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, kFaultWaitEmpty)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full[s], 2u * STAGE_BYTES);
          const uint32_t bar_leader = mapa_shared(smem_u32(&full[s]), 0u);
          issue_half_loads<A_MN, B_MN>(&tma, &tmb, sA + s * A_STAGE_BYTES, sB + s * B_STAGE_BYTES,
                                       bar_leader, m0 + static_cast<int>(rank) * HM,
                                       n0 + static_cast<int>(rank) * HN, kb * BK);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok) {
        if (leader) {
          for (int t = 0; t < STAGES; ++t)
            if (armed & (1u << t)) gemm::drain_wait(&full[t], (armed_par >> t) & 1u);
        }
        settle_inflight_copies();
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t IDESC = make_idesc_bf16_f32(TM, TN, A_MN, B_MN);
      constexpr uint32_t A_KSTEP = A_MN ? UMMA_K * 128 : UMMA_K * 2;
      constexpr uint32_t B_KSTEP = B_MN ? UMMA_K * 128 : UMMA_K * 2;
      constexpr uint32_t A_LBO = A_MN ? MN_CHUNK_BYTES : 16;
      constexpr uint32_t B_LBO = B_MN ? MN_CHUNK_BYTES : 16;
      int s = 0;
      uint32_t ph = 0;
      uint32_t acc = 0, acc_ph = 0;
      bool ok = true;
      Item it;
      for (int i = 0; ok && work_item(i, cluster, num_clusters, num_tiles, p.sk_mode, p.sk_first, k_blocks, it);
           ++i) {
        if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, kFaultWaitAccEmpty)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * TN;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, kFaultWaitFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t ad = make_sw128_desc(a_addr + kk * A_KSTEP, A_LBO, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + kk * B_KSTEP, B_LBO, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, IDESC, (kb != it.kb0 || kk != 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[s], kPairMask);  // frees stage s in both CTAs
          if (++s == STAGES) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair_mc(&acc_full[acc], kPairMask);  // both halves ready for the epilogues
        acc ^= 1u;
        if (acc == 0u) acc_ph ^= 1u;
      }
      umma_commit_pair_mc(drain, 0x1);
      gemm::drain_wait(drain, 0u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const uint32_t q = warp & 3u;                 // TMEM lane quarter
    const uint32_t ew = warp - 2u;                // epilogue warp 0..7
    const int c_lo = static_cast<int>(ew >> 2) * (TN / 64);  // first of this warp's 4 chunks
    uint32_t acc = 0, acc_ph = 0;
    [[maybe_unused]] int pend_region = -1, pend_row = 0, pend_col = 0;
    if constexpr (EPI == kEpiBf16Allreduce) {
      if (blockIdx.x == 0) ar::reduce_db(p, ew, lane);
    }
    Item it;
    for (int i = 0; work_item(i, cluster, num_clusters, num_tiles, p.sk_mode, p.sk_first, k_blocks, it); ++i) {
      const int m0 = (it.tile / n_tiles) * TM + static_cast<int>(rank) * HM;
      const int n0 = (it.tile % n_tiles) * TN;
      if (!mbar_wait(&acc_full[acc], acc_ph, kFaultWaitAccFull)) break;
      tc_fence_after();
      const int row = m0 + static_cast<int>(q * 32 + lane);
      const uint32_t t_row = tmem_base + ((q * 32u) << 16) + acc * TN;
      // Split-K tail: per warp (32 rows) a ticket decides which K half publishes its fp32
      // partial and which one adds it and runs the epilogue. The adder waits only for a
      // partner that already holds its ticket, i.e. is past its main loop.
      bool split = it.split >= 0, adder = false;
      uint32_t word = 0;
      float* part = nullptr;
      if (split) {
        const uint32_t slot = static_cast<uint32_t>(it.split) * 2u + rank;
        word = slot * kEpiWarps + ew;
        part = p.partial + static_cast<size_t>(slot) * (HM * TN) + q * 32u + lane;
        uint32_t t = 0;
        if (lane == 0) t = atomicAdd(&p.tickets[word], 1u);
        adder = __shfl_sync(0xffffffffu, t, 0) != 0u;
        if (adder) {
          uint32_t ok = 1;
          if (lane == 0) ok = wait_ready(&p.ready[word], p.split_wait_ns) ? 1u : 0u;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          uint32_t v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&p.ready[word]) : "memory");
          (void)v;
          if (!ok) part = nullptr;  // partner never published: fault recorded, no add
        }
      }
#pragma unroll 1
      for (int c = c_lo; c < c_lo + TN / 64; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= p.N) break;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_wait_ld();
        if (split && !adder) {
          // partial[col][row] inside the slot: a warp stores 128 contiguous bytes per column
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(part + (c * 32 + j) * HM, __uint_as_float(r[j]));
          continue;
        }
        if (split && part != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __ldcg(part + (c * 32 + j) * HM)));
        }
        gemm::epilogue_chunk<EPI == kEpiBf16Allreduce ? kEpiStoreBf16 : EPI>(p, r, row, col0);
      }
      if (split) {
        __threadfence();
        __syncwarp();
        if (lane == 0) {
          if (!adder) {
            asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&p.ready[word]), "r"(1u) : "memory");
          } else {
            // both halves are done with the words: leave them zero for the next launch
            p.ready[word] = 0u;
            p.tickets[word] = 0u;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0u));
      acc ^= 1u;
      if (acc == 0u) acc_ph ^= 1u;
      if constexpr (EPI == kEpiBf16Allreduce) {
        if (!split || adder) {  // this warp stored its region of the tile on this rank
          const int region = it.tile * ar::kRegionsPerTile + static_cast<int>(rank * 8u + ew);
          ar::signal_region(p, static_cast<uint32_t>(region), lane);
          if (pend_region >= 0) ar::reduce_region(p, static_cast<uint32_t>(pend_region), pend_row, pend_col, lane);
          pend_region = region;
          pend_row = m0 + static_cast<int>(q * 32u);
          pend_col = n0 + c_lo * 32;
        }
      }
    }
    if constexpr (EPI == kEpiBf16Allreduce) {
      if (pend_region >= 0) ar::reduce_region(p, static_cast<uint32_t>(pend_region), pend_row, pend_col, lane);
      ar::finish(p, ew, lane);
    }
  }

  tc_fence_before();
  cluster_sync_all();  // all MMAs complete (leader drained) and both epilogues done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm2
}  // namespace c3cu
