// FlashAttention forward with two query tiles per CTA (ping-pong softmax warpgroups).
//
// Same math, layouts and outputs as flash_fwd_kernel (attn.cu). One CTA owns two adjacent
// 128-row query tiles of one (batch, head), rows [q0, q0 + 256), and streams each K_j / V_j
// block once for both:
//   warp 0      TMA producer: Q0, Q1, then K_j / V_j (128 keys each) into a 2-stage ring
//   warp 1      TMEM owner + MMA issuer, per key block j:
//                 O0 += P0_j V_j, S0_{j+1} = Q0 K_{j+1}^T, O1 += P1_j V_j, S1_{j+1} = Q1 K_{j+1}^T
//               so while warpgroup t turns S_t into P_t, the tensor pipe works on the other
//               tile (two 128x128x128 MMAs, as long as one softmax pass).
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1: one thread per query row, as
//               in flash_fwd_kernel (lazy O rescaling, P written back over S in TMEM).
// TMEM (512 columns): tile t holds S_t / P_t at [256t, 256t + 128) and O_t at
// [256t + 128, 256t + 256). Each tile has a single S buffer: S_t,{j+1} is issued after
// PV_t,j, which reads P_t,j from the same columns; tcgen05.mma operations of one thread
// execute in issue order, so the read precedes the overwrite.
//
// Exponentials all use ex2.approx (MUFU). Moving part of each 32-score chunk to the FMA
// pipe (2^floor(x) times a degree-3 polynomial) measured slower at every fraction tried
// (6, 10, 14, 18 of 32): the softmax is bound by its instruction stream, not by MUFU.
// With 10 warps a sub-partition holds three of them, so its 16K registers cap a thread at
// 168; the 128 scores of a row stay in registers (a three-input max.f32 row maximum made the
// kernel spill at that cap).
#pragma once

namespace c3cu {
namespace attn {

constexpr int kThreads2 = 320;
constexpr int KV_STAGES2 = 2;
// smem: Q0 | Q1 | K0 V0 | K1 V1 | barriers
constexpr uint32_t SMEM_BYTES2 = TILE_BYTES * (2 + 2 * KV_STAGES2) + 16 * 8 + 1024;


__global__ void __launch_bounds__(kThreads2, 1)
    flash_fwd2_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ[2] = {smem, smem + TILE_BYTES};
  uint8_t* sK[KV_STAGES2];
  uint8_t* sV[KV_STAGES2];
  for (int s = 0; s < KV_STAGES2; ++s) {
    sK[s] = smem + TILE_BYTES * (2 + 2 * s);
    sV[s] = smem + TILE_BYTES * (3 + 2 * s);
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TILE_BYTES * (2 + 2 * KV_STAGES2));
  uint64_t* q_full = bars;         // Q0 and Q1
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [tile]
  uint64_t* p_full = bars + 7;     // [tile]
  uint64_t* pv_done = bars + 9;    // [tile]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const uint32_t warp = warp_id_sync();
  const uint32_t lane = lane_id();

  // Head-major order, heaviest causal tile pairs first (as in flash_fwd_kernel).
  const int pairs = (p.q_tiles + 1) / 2;
  const int bh = static_cast<int>(blockIdx.x / pairs);
  const int pr = pairs - 1 - static_cast<int>(blockIdx.x % pairs);
  const int qt0 = 2 * pr;
  const int q0 = qt0 * BM;
  const bool v1 = qt0 + 1 < p.q_tiles;  // the second tile has rows
  const int kv_blocks_total = (p.S + BN - 1) / BN;
  const int n0 = p.causal ? min(qt0 + 1, kv_blocks_total) : kv_blocks_total;
  const int n1 = v1 ? (p.causal ? min(qt0 + 2, kv_blocks_total) : kv_blocks_total) : 0;
  const int nkv = max(n0, n1);

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbarrier_init();
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      bool ok = true;
      mbar_arrive_expect_tx(q_full, (v1 ? 2u : 1u) * TILE_BYTES);
      tma_load_3d(sQ[0], &tmq, q_full, 0, q0, bh);
      tma_load_3d(sQ[0] + BOX_BYTES, &tmq, q_full, 64, q0, bh);
      if (v1) {
        tma_load_3d(sQ[1], &tmq, q_full, 0, q0 + BM, bh);
        tma_load_3d(sQ[1] + BOX_BYTES, &tmq, q_full, 64, q0 + BM, bh);
      }
      for (int j = 0; j < nkv; ++j) {
        const int st = j % KV_STAGES2;
        const uint32_t ph = (j / KV_STAGES2) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, kFaultWaitEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        const int k0 = j * BN;
        tma_load_3d(sK[st], &tmk, &kv_full[st], 0, k0, bh);
        tma_load_3d(sK[st] + BOX_BYTES, &tmk, &kv_full[st], 64, k0, bh);
        tma_load_3d(sV[st], &tmv, &kv_full[st], 0, k0, bh);
        tma_load_3d(sV[st] + BOX_BYTES, &tmv, &kv_full[st], 64, k0, bh);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      drain_wait(q_full, 0u);
      if (!ok)
        for (int t = 0; t < KV_STAGES2; ++t)
          if (armed & (1u << t)) drain_wait(&kv_full[t], (armed_par >> t) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = make_idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_PV = make_idesc_bf16_f32(BM, HD, false, true);
      auto kv_ready = [&](int j) -> bool {
        const int st = j % KV_STAGES2;
        if (!mbar_wait(&kv_full[st], (j / KV_STAGES2) & 1u, kFaultWaitFull)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int t, int j) {
        const int st = j % KV_STAGES2;
        const uint32_t qa = smem_u32(sQ[t]), ka = smem_u32(sK[st]);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk / 4) * BOX_BYTES + (kk % 4) * 32;
          umma_f16_ss(tmem + 256u * t, make_sw128_desc(qa + off, 16, 1024),
                      make_sw128_desc(ka + off, 16, 1024), IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const int st = j % KV_STAGES2;
        const uint32_t va = smem_u32(sV[st]);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16_ts(tmem + 256u * t + 128u, tmem + 256u * t + kk * 8,
                      make_sw128_desc(va + kk * 2048, BOX_BYTES, 1024), IDESC_PV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[t]);
      };
      bool ok = mbar_wait(q_full, 0u, kFaultWaitFull);
      if (ok && nkv > 0) ok = kv_ready(0);
      if (ok && n0 > 0) issue_s(0, 0);
      if (ok && n1 > 0) issue_s(1, 0);
      for (int j = 0; j < nkv && ok; ++j) {
        bool next_ready = false;
        if (j < n0) {
          if (!mbar_wait(&p_full[0], j & 1u, kFaultWaitSoftmax)) { ok = false; break; }
          tc_fence_after();
          issue_pv(0, j);
          if (j + 1 < n0) {
            if (!kv_ready(j + 1)) { ok = false; break; }
            next_ready = true;
            issue_s(0, j + 1);
          }
        }
        if (j < n1) {
          if (!mbar_wait(&p_full[1], j & 1u, kFaultWaitSoftmax)) { ok = false; break; }
          tc_fence_after();
          issue_pv(1, j);
          if (j + 1 < n1) {
            if (!next_ready && !kv_ready(j + 1)) { ok = false; break; }
            issue_s(1, j + 1);
          }
        }
        umma_commit(&kv_empty[j % KV_STAGES2]);  // stage free once block j's MMAs are done
      }
      umma_commit(drain);
      drain_wait(drain, 0u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax (warps 2..9)
    const int t = static_cast<int>((warp - 2u) >> 2);  // query tile of this warpgroup
    const uint32_t q = warp & 3u;                      // TMEM lane quarter
    const uint32_t lane_base = (q * 32u) << 16;
    const uint32_t s_base = tmem + lane_base + 256u * t;
    const uint32_t o_base = s_base + 128u;
    const int row = q0 + t * BM + static_cast<int>(q * 32 + lane);
    const int n = t == 0 ? n0 : n1;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[t], j & 1u, kFaultWaitAccFull)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(s_base + c * 32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
      }
      tmem_wait_ld();
      const int k0 = j * BN;
      if ((p.causal && k0 + BN - 1 > row) || (k0 + BN > p.S)) {
        const int lim = p.causal ? min(row, p.S - 1) : p.S - 1;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (k0 + i > lim) s[i] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1];
#pragma unroll
      for (int i = 2; i < 128; i += 2) {
        mx0 = fmaxf(mx0, s[i]);
        mx1 = fmaxf(mx1, s[i + 1]);
      }
      const float m_new = fmaxf(m_used, fmaxf(mx0, mx1) * p.scale_log2);
      const bool need = (m_used == -INFINITY) ? (m_new != -INFINITY) : (m_new > m_used + kRescaleThreshold);
      const float m_next = need ? m_new : m_used;
      const float alpha = need ? ((m_used == -INFINITY) ? 0.f : ex2(m_used - m_new)) : 1.f;
      const float base = (m_next == -INFINITY) ? 0.f : m_next;
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 nb2 = make_float2(-base, -base);
      float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float2 x = make_float2(s[c * 32 + 2 * i], s[c * 32 + 2 * i + 1]);
          x = ffma2(x, sc2, nb2);
          const float2 e = make_float2(ex2(x.x), ex2(x.y));
          rs2 = fadd2(rs2, e);
          w[i] = pack_bf16x2(e.x, e.y);
        }
        tmem_st_32x32b_x16(s_base + c * 16, w);
      }
      const float rs = rs2.x + rs2.y;
      l = l * alpha + rs;
      // Rescaling O needs PV_{t,j-1} complete. S_{t,j} was issued after it in the same
      // in-order MMA stream and has completed, so this wait returns at once; it documents
      // (and enforces) the ordering.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        if (!mbar_wait(&pv_done[t], (j - 1) & 1u, kFaultWaitAccFull)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(o_base + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) { lo[i] = r[i]; hi[i] = r[16 + i]; }
          tmem_st_32x32b_x16(o_base + c * 32, lo);
          tmem_st_32x32b_x16(o_base + c * 32 + 16, hi);
        }
      }
      m_used = m_next;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && n > 0 && mbar_wait(&pv_done[t], (n - 1) & 1u, kFaultWaitAccFull)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.O + (static_cast<int64_t>(bh) * p.S + row) * HD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(o_base + c * 32, r);
        tmem_wait_ld();
        if (row < p.S) {
          uint4* o4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            o4[v] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * v]) * inv, __uint_as_float(r[8 * v + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv));
        }
      }
      if (row < p.S && p.lse)
        p.lse[static_cast<int64_t>(bh) * p.S + row] =
            (l > 0.f) ? (m_used * 0.69314718055994530942f + logf(l)) : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn
}  // namespace c3cu
