// Causal (or full) FlashAttention forward on the 5th-generation tensor cores (tcgen05).
// The reference has no attention kernel; this implements O = softmax(scale * Q K^T + mask) V
// and LSE = log(sum exp(scale * Q K^T + mask)) (natural log) for bf16 Q, K, V of shape
// [B, H, S, D=128] and fp32 LSE [B, H, S].
//
// One CTA per 128-row query tile (grid = B*H*ceil(S/128), head-major, heaviest tiles first):
//   warp 0      TMA producer: Q once, then K_j / V_j (128 keys each) into a 2-stage ring
//   warp 1      TMEM owner + MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers
//               (issued one block ahead, so it overlaps the softmax of the previous block),
//               then O += P_j V_j with P_j read from TMEM (A operand) and V_j MN-major
//   warps 2..5  softmax, one thread per query row: tcgen05.ld of its S row (thread-local
//               row maximum), exp2 in fp32, row sum, P_j packed to bf16 and written back into
//               the S buffer; O is rescaled in TMEM only when the running maximum grows by
//               more than 2^8 (lazy rescaling), and normalised by the row sum at the end
// TMEM: S buffers at columns [0,128) and [128,256), O at [256,384) (512 allocated).
// The default launch is flash_fwd3_kernel (attn3.cuh): two query tiles per CTA sharing each
// 64-key K / V block, two S buffers per tile, ping-pong softmax warpgroups. flash_fwd2_kernel
// (attn2.cuh, 128-key blocks, one S buffer per tile) is variant 2 and this single-tile kernel
// variant 1. Variant 4 is flash_fwd3_kernel<true>: the same computation with the two tiles'
// softmax warps of each SM sub-partition taking turns at their exponentials (experimental).
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>

#include "common.cuh"
#include "host_util.h"

C3CU_FAULT_ACCESSORS(attn)

namespace c3cu {
namespace attn {

constexpr int BM = 128;                        // query rows per CTA
constexpr int BN = 128;                        // keys per block
constexpr int HD = 128;                        // head dim
constexpr int kThreads = 192;
constexpr uint32_t BOX_BYTES = 128 * 64 * 2;   // one TMA box: 128 rows x 64 bf16 (16 KiB)
constexpr uint32_t TILE_BYTES = 2 * BOX_BYTES; // a 128 x 128 bf16 tile as two 64-column boxes
constexpr int KV_STAGES = 2;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 256;
__host__ __device__ constexpr uint32_t s_col(int j) { return (j & 1) ? 128u : 0u; }
constexpr float kRescaleThreshold = 8.0f;      // log2 units: P stays <= 2^8 between rescales
// smem: Q | K0 V0 | K1 V1 | barriers
constexpr uint32_t SMEM_BYTES = TILE_BYTES * (1 + 2 * KV_STAGES) + 16 * 8 + 1024;

struct Params {
  int BH;                 // batch * heads
  int S;                  // sequence length
  int q_tiles;            // ceil(S / 128)
  float scale_log2;       // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* O;       // [BH][S][128]
  float* lse;             // [BH][S]
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-lane fp32 arithmetic (sm_100): halves the FMA-pipe instructions of the softmax.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(reinterpret_cast<uint64_t&>(d))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)),
        "l"(reinterpret_cast<const uint64_t&>(c)));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(reinterpret_cast<uint64_t&>(d))
      : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
  return d;
}

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

__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK[KV_STAGES];
  uint8_t* sV[KV_STAGES];
  for (int s = 0; s < KV_STAGES; ++s) {
    sK[s] = smem + TILE_BYTES * (1 + 2 * s);
    sV[s] = smem + TILE_BYTES * (2 + 2 * s);
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TILE_BYTES * (1 + 2 * KV_STAGES));
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* p_full = bars + 7;     // [2]
  uint64_t* pv_done = bars + 9;    // [2]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const uint32_t warp = warp_id_sync();
  const uint32_t lane = lane_id();

  // Head-major order: the CTAs resident at one time share a few heads, so their K / V blocks
  // are read from HBM once and then hit in L2; within a head the heaviest causal tiles
  // (most key blocks) come first.
  const int bh = static_cast<int>(blockIdx.x / p.q_tiles);
  const int qt = p.q_tiles - 1 - static_cast<int>(blockIdx.x % p.q_tiles);
  const int q0 = qt * BM;
  const int kv_blocks_total = (p.S + BN - 1) / BN;
  const int n = p.causal ? min(qt + 1, kv_blocks_total) : kv_blocks_total;

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
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_3d(sQ, &tmq, q_full, 0, q0, bh);
      tma_load_3d(sQ + BOX_BYTES, &tmq, q_full, 64, q0, bh);
      for (int j = 0; j < n; ++j) {
        const int st = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1u;
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
      // every copy this lane issued lands before the CTA exits (normal and fault paths)
      drain_wait(q_full, 0u);
      if (!ok)
        for (int t = 0; t < KV_STAGES; ++t)
          if (armed & (1u << t)) drain_wait(&kv_full[t], (armed_par >> t) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // S = Q K^T: A = Q (K-major over d), B = K tile (K-major over d), M = N = 128
      constexpr uint32_t IDESC_QK = make_idesc_bf16_f32(BM, BN, false, false);
      // O += P V: A = P from TMEM, B = V tile (MN-major: d contiguous), N = 128 (d), K = keys
      constexpr uint32_t IDESC_PV = make_idesc_bf16_f32(BM, HD, false, true);
      bool ok = mbar_wait(q_full, 0u, kFaultWaitFull);
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&kv_full[st], (j / KV_STAGES) & 1u, kFaultWaitFull)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK[st]);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk / 4) * BOX_BYTES + (kk % 4) * 32;
          umma_f16_ss(tmem + s_col(j), make_sw128_desc(qa + off, 16, 1024),
                      make_sw128_desc(ka + off, 16, 1024), IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) {
          // S buffer (j+1)&1 held P_{j-1}: wait until PV_{j-1} has read it
          if (j >= 1 && !mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) / 2) & 1u, kFaultWaitAccEmpty)) {
            ok = false;
            break;
          }
          if (!issue_s(j + 1)) { ok = false; break; }
        }
        if (!mbar_wait(&p_full[j & 1], (j / 2) & 1u, kFaultWaitSoftmax)) { ok = false; break; }
        tc_fence_after();
        const int st = j % KV_STAGES;
        const uint32_t va = smem_u32(sV[st]);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A: P columns (2 bf16 per 32-bit column), 16 keys = 8 columns per step
          // B: V rows = keys: 16 keys x 128 B = 2 KiB per step; the two d halves 16 KiB apart
          umma_f16_ts(tmem + O_COL, tmem + s_col(j) + kk * 8,
                      make_sw128_desc(va + kk * 2048, BOX_BYTES, 1024), IDESC_PV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[j & 1]);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(drain);
      drain_wait(drain, 0u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax (warps 2..5)
    const uint32_t q = warp & 3u;
    const uint32_t lane_base = (q * 32u) << 16;
    const int row = q0 + static_cast<int>(q * 32 + lane);
    float m_used = -INFINITY;  // log2-domain running maximum P is taken against
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j / 2) & 1u, kFaultWaitAccFull)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_base + s_col(j) + c * 32, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
      }
      tmem_wait_ld();
      const int k0 = j * BN;
      // Masking (causal, or keys past the sequence end) only on edge blocks, outside the
      // common path. The scale is positive, so the row maximum is taken on raw scores.
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
      // e = 2^(s * scale_log2 - base): one packed FMA per pair, then ex2
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 nb2 = make_float2(-base, -base);
      float2 rs2 = make_float2(0.f, 0.f);
      // P_j (bf16, relative to m_next) overwrites the first 64 columns of this S buffer;
      // chunk c (keys 32c..32c+31) lands in columns 16c..16c+15, already read above.
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
        tmem_st_32x32b_x16(tmem + lane_base + s_col(j) + c * 16, w);
      }
      const float rs = rs2.x + rs2.y;
      l = l * alpha + rs;
      // O may only be rescaled once PV_{j-1} has completed. P_j goes to the other S buffer
      // and PV_j is issued after PV_{j-1} by the same thread (tcgen05.mma executes in issue
      // order), so without a rescale the softmax does not wait for PV_{j-1}.
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) / 2) & 1u, kFaultWaitAccFull)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) { lo[i] = r[i]; hi[i] = r[16 + i]; }
          tmem_st_32x32b_x16(tmem + lane_base + O_COL + c * 32, lo);
          tmem_st_32x32b_x16(tmem + lane_base + O_COL + c * 32 + 16, hi);
        }
      }
      m_used = m_next;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j & 1]);
    }
    if (ok && n > 0 && mbar_wait(&pv_done[(n - 1) & 1], ((n - 1) / 2) & 1u, kFaultWaitAccFull)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.O + (static_cast<int64_t>(bh) * p.S + row) * HD;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, r);
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

#include "attn2.cuh"
#include "attn3.cuh"

namespace c3cu {
namespace attn {

// 0 = automatic (= 3), 1 = one query tile per CTA, 2 = two query tiles with 128-key blocks,
// 3 = two query tiles with 64-key blocks and two S buffers per tile.
static std::atomic<int> g_attn_variant{0};  // process-wide; set by c3cu_set_attn_variant

namespace {
int encode_bhsd(CUtensorMap* map, const void* base, int64_t BH, int64_t S, uint32_t box_rows = 128) {
  if (!aligned16(base)) {
    set_error("flash_attn_fwd: tensor base %p is not 16-byte aligned", base);
    return C3CU_ERR_ALIGN;
  }
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
            cudaSuccess || q != cudaDriverEntryPointSuccess) {
      set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
      return C3CU_ERR_CUDA;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(HD), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(HD) * 2, static_cast<cuuint64_t>(S) * HD * 2};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("flash_attn_fwd: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return C3CU_ERR_CUDA;
  }
  return C3CU_OK;
}
}  // namespace

}  // namespace attn
}  // namespace c3cu

extern "C" int c3cu_flash_attn_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE,
                                   int64_t B, int64_t H, int64_t S, int64_t D, float scale, int causal,
                                   c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (B < 0 || H < 0 || S < 0 || B * H > INT32_MAX || S > INT32_MAX) {
    set_error("flash_attn_fwd: sizes out of range");
    return C3CU_ERR_INVALID;
  }
  if (D != attn::HD) {
    set_error("flash_attn_fwd: head dim %lld is not supported (128 only)", (long long)D);
    return C3CU_ERR_INVALID;
  }
  if (B * H == 0 || S == 0) return C3CU_OK;
  if (!Q || !K || !V || !O) {
    set_error("flash_attn_fwd: null tensor");
    return C3CU_ERR_INVALID;
  }
  CUtensorMap tq, tk, tv;
  if ((rc = attn::encode_bhsd(&tq, Q, B * H, S)) != C3CU_OK) return rc;
  if ((rc = attn::encode_bhsd(&tk, K, B * H, S)) != C3CU_OK) return rc;
  if ((rc = attn::encode_bhsd(&tv, V, B * H, S)) != C3CU_OK) return rc;
  if (!aligned16(O)) {
    set_error("flash_attn_fwd: output is not 16-byte aligned");
    return C3CU_ERR_ALIGN;
  }
  attn::Params p;
  p.BH = static_cast<int>(B * H);
  p.S = static_cast<int>(S);
  p.q_tiles = static_cast<int>((S + attn::BM - 1) / attn::BM);
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634074);
  p.causal = causal ? 1 : 0;
  p.O = static_cast<__nv_bfloat16*>(O);
  p.lse = LSE;
  const int variant = attn::g_attn_variant.load(std::memory_order_relaxed);  // one value for the whole call
  if (variant == 1) {
    static std::atomic<uint64_t> smem_set{0};
    rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn::flash_fwd_kernel), attn::SMEM_BYTES,
                              smem_set, "flash_attn_fwd: set shared memory");
    if (rc != C3CU_OK) return rc;
    const int64_t grid = static_cast<int64_t>(p.BH) * p.q_tiles;
    if (grid > INT32_MAX) {
      set_error("flash_attn_fwd: grid too large");
      return C3CU_ERR_INVALID;
    }
    attn::flash_fwd_kernel<<<static_cast<unsigned>(grid), attn::kThreads, attn::SMEM_BYTES,
                             static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
    return cuda_status(cudaGetLastError(), "flash_attn_fwd: launch");
  }
  const int64_t grid = static_cast<int64_t>(p.BH) * ((p.q_tiles + 1) / 2);
  if (grid > INT32_MAX) {
    set_error("flash_attn_fwd: grid too large");
    return C3CU_ERR_INVALID;
  }
  if (variant == 0 || variant == 3 || variant == 4) {
    // 64-key blocks: K / V tensor maps with 64-row boxes
    CUtensorMap tk64, tv64;
    if ((rc = attn::encode_bhsd(&tk64, K, B * H, S, 64)) != C3CU_OK) return rc;
    if ((rc = attn::encode_bhsd(&tv64, V, B * H, S, 64)) != C3CU_OK) return rc;
    if (variant == 4) {
      static std::atomic<uint64_t> smem_set4{0};
      rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn::flash_fwd3_kernel<true>), attn::SMEM_BYTES3,
                                smem_set4, "flash_attn_fwd: set shared memory");
      if (rc != C3CU_OK) return rc;
      attn::flash_fwd3_kernel<true><<<static_cast<unsigned>(grid), attn::kThreads3, attn::SMEM_BYTES3,
                                      static_cast<cudaStream_t>(stream)>>>(tq, tk64, tv64, p);
      return cuda_status(cudaGetLastError(), "flash_attn_fwd: launch");
    }
    static std::atomic<uint64_t> smem_set3{0};
    rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn::flash_fwd3_kernel<false>), attn::SMEM_BYTES3,
                              smem_set3, "flash_attn_fwd: set shared memory");
    if (rc != C3CU_OK) return rc;
    attn::flash_fwd3_kernel<false><<<static_cast<unsigned>(grid), attn::kThreads3, attn::SMEM_BYTES3,
                                     static_cast<cudaStream_t>(stream)>>>(tq, tk64, tv64, p);
    return cuda_status(cudaGetLastError(), "flash_attn_fwd: launch");
  }
  static std::atomic<uint64_t> smem_set2{0};
  rc = set_max_dynamic_smem(reinterpret_cast<const void*>(attn::flash_fwd2_kernel), attn::SMEM_BYTES2,
                            smem_set2, "flash_attn_fwd: set shared memory");
  if (rc != C3CU_OK) return rc;
  attn::flash_fwd2_kernel<<<static_cast<unsigned>(grid), attn::kThreads2, attn::SMEM_BYTES2,
                            static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return cuda_status(cudaGetLastError(), "flash_attn_fwd: launch");
}

extern "C" int c3cu_set_attn_variant(int variant) {
  if (variant < 0 || variant > 4) {
    c3cu::set_error("set_attn_variant: unknown variant %d", variant);
    return C3CU_ERR_INVALID;
  }
  c3cu::attn::g_attn_variant.store(variant, std::memory_order_relaxed);
  return C3CU_OK;
}
