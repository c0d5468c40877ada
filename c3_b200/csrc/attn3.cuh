// FlashAttention forward, two query tiles per CTA, 64-key blocks with S double-buffered per
// tile (variant 3).
//
// Same math, layouts and outputs as flash_fwd2_kernel. With 128-key blocks each tile's TMEM
// (S 128 + O 128 columns, two tiles = 512) holds a single S buffer, so a tile's next QK^T can
// only start after its softmax and its P V: the tile's period is the softmax latency plus two
// MMAs. With 64-key blocks a tile holds two S buffers of 64 columns and O (64 + 64 + 128 = 256
// columns), and the MMA warp keeps S_{t,j+2} in flight while the softmax works on block j:
//   TMEM tile t: S buffers at 256t + {0, 64}, O at 256t + 128.
//   warp 0      TMA: Q0, Q1 (128 rows each), then K_j / V_j (64 keys) into a 4-stage ring
//   warp 1      MMA: for j, tile t: O_t += P_{t,j} V_j, then S_{t,j+2} = Q_t K_{j+2}^T into
//               the buffer P_{t,j} came from (tcgen05.mma ops of one thread run in order)
//   warps 2..5  softmax of tile 0, warps 6..9 of tile 1 (one thread per row, 64 scores).
//
// ALT (variant 4): warps 2+i and 6+i (i = 0..3) share an SM sub-partition and its MUFU unit.
// Left alone they reach their exponentials at about the same time, so the exponentials of both
// tiles contend while the TMEM loads, row maxima and P stores of both wait at once. With ALT the
// two take turns: a warp runs the exponentials of its block only after its partner has finished
// the partner's previous exponentials (tile 0 goes first), through a token mbarrier per warp
// (bounded waits; a warp stops waiting once its partner has finished all its blocks, as the
// causal tiles have different block counts).
#pragma once

namespace c3cu {
namespace attn {

constexpr int BKV3 = 64;                          // keys per block
constexpr uint32_t KV_BOX3 = 64 * 64 * 2;         // one TMA box: 64 keys x 64 d (8 KiB)
constexpr uint32_t KV_TILE3 = 2 * KV_BOX3;        // K_j or V_j: 64 keys x 128 d
constexpr int KV_STAGES3 = 4;
constexpr int kThreads3 = 320;
// smem: Q0 | Q1 | (K V) x stages | barriers
constexpr uint32_t SMEM_BYTES3 = 2 * TILE_BYTES + KV_STAGES3 * 2 * KV_TILE3 + 32 * 8 + 1024;

// Waits for a token mbarrier phase, or until the partner warp has set its done flag (it has no
// more tokens to hand over). Bounded: records kFaultWaitSoftmax and returns false at the limit.
__device__ __forceinline__ bool token_wait(uint64_t* bar, uint32_t parity, const volatile int* partner_done) {
  if (mbar_try_wait(bar, parity) || *partner_done) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity) || *partner_done) return true;
    if ((++spins & 255u) == 0u) {
      if (fault_raised()) return false;
      if (globaltimer_ns() - t0 > C3CU_WAIT_LIMIT_NS) {
        record_fault(kFaultWaitSoftmax, blockIdx.x & 0xffffu);
        return false;
      }
    }
  }
}

template <bool ALT>
__global__ void __launch_bounds__(kThreads3, 1)
    flash_fwd3_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ[2] = {smem, smem + TILE_BYTES};
  uint8_t* sK[KV_STAGES3];
  uint8_t* sV[KV_STAGES3];
  for (int s = 0; s < KV_STAGES3; ++s) {
    sK[s] = smem + 2 * TILE_BYTES + s * 2 * KV_TILE3;
    sV[s] = sK[s] + KV_TILE3;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * TILE_BYTES + KV_STAGES3 * 2 * KV_TILE3);
  uint64_t* q_full = bars;                       // 1
  uint64_t* kv_full = bars + 1;                  // [stages]
  uint64_t* kv_empty = kv_full + KV_STAGES3;     // [stages]
  uint64_t* s_full = kv_empty + KV_STAGES3;      // [tile][buffer]
  uint64_t* p_full = s_full + 4;                 // [tile]
  uint64_t* pv_done = p_full + 2;                // [tile]
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // ALT only: token[4 * t + i] is handed to tile t's warp of pair i; done[4 * t + i] is set once
  // that warp has run its last block (bytes 152..247 of the 256 reserved for barriers)
  uint64_t* token = drain + 2;
  int* done = reinterpret_cast<int*>(token + 8);

  const uint32_t warp = warp_id_sync();
  const uint32_t lane = lane_id();

  const int pairs = (p.q_tiles + 1) / 2;
  const int bh = static_cast<int>(blockIdx.x / pairs);
  const int pr = pairs - 1 - static_cast<int>(blockIdx.x % pairs);
  const int qt0 = 2 * pr;
  const int q0 = qt0 * BM;
  const bool v1 = qt0 + 1 < p.q_tiles;
  const int kv_total = (p.S + BKV3 - 1) / BKV3;
  const int n0 = p.causal ? min(2 * (qt0 + 1), kv_total) : kv_total;
  const int n1 = v1 ? (p.causal ? min(2 * (qt0 + 2), kv_total) : kv_total) : 0;
  const int nkv = max(n0, n1);

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KV_STAGES3; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&s_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    if constexpr (ALT) {
      for (int i = 0; i < 8; ++i) {
        mbar_init(&token[i], 1);
        done[i] = 0;
      }
    }
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
        const int st = j % KV_STAGES3;
        const uint32_t ph = (j / KV_STAGES3) & 1u;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, kFaultWaitEmpty)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[st], 2 * KV_TILE3);
        const int k0 = j * BKV3;
        tma_load_3d(sK[st], &tmk, &kv_full[st], 0, k0, bh);
        tma_load_3d(sK[st] + KV_BOX3, &tmk, &kv_full[st], 64, k0, bh);
        tma_load_3d(sV[st], &tmv, &kv_full[st], 0, k0, bh);
        tma_load_3d(sV[st] + KV_BOX3, &tmv, &kv_full[st], 64, k0, bh);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      drain_wait(q_full, 0u);
      if (!ok)
        for (int t = 0; t < KV_STAGES3; ++t)
          if (armed & (1u << t)) drain_wait(&kv_full[t], (armed_par >> t) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = make_idesc_bf16_f32(BM, BKV3, false, false);
      constexpr uint32_t IDESC_PV = make_idesc_bf16_f32(BM, HD, false, true);
      int kv_waited = -1;  // highest block whose K/V arrival has been observed
      auto kv_ready = [&](int j) -> bool {
        for (int b = kv_waited + 1; b <= j; ++b) {
          if (!mbar_wait(&kv_full[b % KV_STAGES3], (b / KV_STAGES3) & 1u, kFaultWaitFull)) return false;
          kv_waited = b;
        }
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int t, int j) {
        const int st = j % KV_STAGES3;
        const uint32_t qa = smem_u32(sQ[t]), ka = smem_u32(sK[st]);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qoff = (kk / 4) * BOX_BYTES + (kk % 4) * 32;
          const uint32_t koff = (kk / 4) * KV_BOX3 + (kk % 4) * 32;
          umma_f16_ss(tmem + 256u * t + 64u * (j & 1), make_sw128_desc(qa + qoff, 16, 1024),
                      make_sw128_desc(ka + koff, 16, 1024), IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[2 * t + (j & 1)]);
      };
      auto issue_pv = [&](int t, int j) {
        const int st = j % KV_STAGES3;
        const uint32_t va = smem_u32(sV[st]);
#pragma unroll
        for (int kk = 0; kk < BKV3 / 16; ++kk)
          umma_f16_ts(tmem + 256u * t + 128u, tmem + 256u * t + 64u * (j & 1) + kk * 8,
                      make_sw128_desc(va + kk * 2048, KV_BOX3, 1024), IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[t]);
      };
      const int n_t[2] = {n0, n1};
      bool ok = mbar_wait(q_full, 0u, kFaultWaitFull);
      // prologue: the first two blocks' scores of both tiles
      for (int j = 0; j < 2 && ok; ++j)
        for (int t = 0; t < 2; ++t)
          if (j < n_t[t]) {
            if (!kv_ready(j)) { ok = false; break; }
            issue_s(t, j);
          }
      for (int j = 0; j < nkv && ok; ++j) {
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= n_t[t]) continue;
          if (!mbar_wait(&p_full[t], j & 1u, kFaultWaitSoftmax)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 2 < n_t[t]) {
            if (!kv_ready(j + 2)) { ok = false; break; }
            issue_s(t, j + 2);  // into the buffer P_{t,j} was read from: after issue_pv in order
          }
        }
        umma_commit(&kv_empty[j % KV_STAGES3]);
      }
      umma_commit(drain);
      drain_wait(drain, 0u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax (warps 2..9)
    const int t = static_cast<int>((warp - 2u) >> 2);
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = (q * 32u) << 16;
    const uint32_t t_base = tmem + lane_base + 256u * t;
    const uint32_t o_base = t_base + 128u;
    const int row = q0 + t * BM + static_cast<int>(q * 32 + lane);
    const int n = t == 0 ? n0 : n1;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    // ALT: this warp's token and its partner's (the other tile's warp on the same sub-partition)
    [[maybe_unused]] const uint32_t pair = warp & 3u;
    [[maybe_unused]] uint64_t* my_token = token + 4 * t + pair;
    [[maybe_unused]] uint64_t* partner_token = token + 4 * (1 - t) + pair;
    [[maybe_unused]] const volatile int* partner_done = done + 4 * (1 - t) + pair;
    for (int j = 0; j < n; ++j) {
      const uint32_t s_base = t_base + 64u * (j & 1);
      if (!mbar_wait(&s_full[2 * t + (j & 1)], (j >> 1) & 1u, kFaultWaitAccFull)) { ok = false; break; }
      tc_fence_after();
      float s[BKV3];
#pragma unroll
      for (int c = 0; c < BKV3 / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(s_base + c * 32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
      }
      tmem_wait_ld();
      const int k0 = j * BKV3;
      if ((p.causal && k0 + BKV3 - 1 > row) || (k0 + BKV3 > p.S)) {
        const int lim = p.causal ? min(row, p.S - 1) : p.S - 1;
#pragma unroll
        for (int i = 0; i < BKV3; ++i)
          if (k0 + i > lim) s[i] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1];
#pragma unroll
      for (int i = 2; i < BKV3; i += 2) {
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
      if constexpr (ALT) {
        // tile 0's exponentials of block j follow tile 1's of block j - 1; tile 1's of block j
        // follow tile 0's of block j (token phase = number of the partner's finished turns - 1)
        const bool first = t == 0 && j == 0;
        if (!first && !token_wait(my_token, static_cast<uint32_t>(t == 0 ? j - 1 : j) & 1u, partner_done)) {
          ok = false;
          break;
        }
      }
#pragma unroll
      for (int c = 0; c < BKV3 / 32; ++c) {
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
      if constexpr (ALT) {
        __syncwarp();
        if (lane == 0) mbar_arrive(partner_token);  // the partner's turn
      }
      l = l * alpha + (rs2.x + rs2.y);
      // Rescaling O needs PV_{t,j-1} complete; unlike the single-buffer kernel, S_{t,j} was
      // issued before PV_{t,j-1}, so this wait can block.
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
      // p_full[t] must not run two phases ahead of the MMA warp (its parity wait would miss
      // a phase): release block j only once PV_{t,j-1} is complete, which the MMA issues
      // after consuming phase j-1. In steady state it finished long before.
      if (j > 0 && !mbar_wait(&pv_done[t], (j - 1) & 1u, kFaultWaitAccFull)) { ok = false; break; }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if constexpr (ALT) {
      // no more turns from this warp: its partner stops waiting for them
      __syncwarp();
      if (lane == 0) *reinterpret_cast<volatile int*>(done + 4 * t + pair) = 1;
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
