// In-switch (NVLink SHARP) all-reduce of an fp32 buffer held in multicast-mapped memory.
//
// Every rank's buffer is bound to one NVLink multicast object. Rank r owns slice r of the
// buffer: it loads that slice through the multicast address with multimem.ld_reduce (the
// NVSwitch returns the sum over all ranks) and writes the sum back with multimem.st (the
// switch writes it into every rank's copy). Per rank, one buffer's worth of data crosses
// NVLink in each direction, and the reduction itself costs no SM arithmetic.
//
// Ordering: a rank may read peers' data only after every peer has finished writing it, and
// the result may be consumed only after every rank has stored its slice. Both points are
// grid-wide, cross-GPU barriers on a counter that lives in the same multicast buffer:
// multimem.red.release adds 1 to every rank's copy of the counter, and each CTA spins
// (bounded by %globaltimer) with acquire loads on its local copy until all ranks have
// arrived. The counter only grows: call e (0-based, the same on every rank) waits for
// world * (2e + 1) and world * (2e + 2).
//
// No TMA and no multicast TMA loads are used; only multimem loads/stores/reductions, and (in
// the split call) plain 16-byte loads of each rank's copy through its unicast address.
#include <atomic>
#include <utility>

#include "common.cuh"
#include "host_util.h"
#include "multimem.cuh"

C3CU_FAULT_ACCESSORS(nvls)

namespace c3cu {
namespace nvls {

constexpr int kThreads = 512;
// Switch round trips in flight per thread (multimem.ld_reduce has a long latency: the switch
// gathers from every GPU).
#ifndef C3CU_NVLS_UNROLL
#define C3CU_NVLS_UNROLL 8
#endif
constexpr int kUnroll = C3CU_NVLS_UNROLL;

// CTAs per thread-block cluster of the all-reduce launches (c3cu_set_collective_cluster): 1, or
// 2 so that each pair of CTAs takes both SMs of one TPC and leaves whole TPCs to a CTA-pair GEMM
// running beside it.
std::atomic<int> g_cluster{1};

template <typename... KArgs, typename... Args>
cudaError_t launch_ar(void (*kern)(KArgs...), int num_ctas, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(num_ctas));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  const int cl = g_cluster.load(std::memory_order_relaxed);
  if (cl > 1 && num_ctas % cl == 0) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

using mm::ld_acquire_sys;
using mm::ld_reduce_bf16x8;
using mm::ld_reduce_f32;
using mm::ld_reduce_f32x4;
using mm::red_release_add;
using mm::st_bf16x8;
using mm::st_f32;
using mm::st_f32x4;

// Grid-wide cross-rank barrier: every CTA adds 1 through the multicast address, then waits
// until all world * gridDim.x arrivals of this phase are visible in the local copy.
__device__ bool barrier(uint32_t* mc_flag, const uint32_t* local_flag, uint32_t target) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    red_release_add(mc_flag, 1u);
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(local_flag) - target) < 0) {
      if (globaltimer_ns() - t0 > C3CU_WAIT_LIMIT_NS / 2) {
        record_fault(kFaultWaitPeer, blockIdx.x & 0xffffu);
        ok = false;
        break;
      }
    }
  }
  __syncthreads();
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// Reduces this rank's slice of a segment of `count` elements at `mc` (16-byte units of
// kPerVec elements; count must be a multiple of kPerVec).
// The work is spread over CTAs [0, nctas) of the grid; `cta` is this CTA's index among them.
template <bool BF16>
__device__ __forceinline__ void reduce_segment(uint8_t* mc, int64_t count, int rank, int world, int cta,
                                               int nctas) {
  constexpr int64_t kPerVec = BF16 ? 8 : 4;
  const int64_t nvec = count / kPerVec;
  const int64_t per = (nvec + world - 1) / world;
  const int64_t v0 = per * rank;
  const int64_t v1 = min(nvec, v0 + per);
  const int64_t stride = static_cast<int64_t>(nctas) * blockDim.x;
  int64_t i = v0 + static_cast<int64_t>(cta) * blockDim.x + threadIdx.x;
  for (; i + stride * (kUnroll - 1) < v1; i += stride * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint8_t* a = mc + (i + stride * u) * 16;
      if (BF16) {
        ld_reduce_bf16x8(a, v[u]);
      } else {
        float4 f;
        ld_reduce_f32x4(reinterpret_cast<float*>(a), f);
        v[u] = make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z), __float_as_uint(f.w));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      uint8_t* a = mc + (i + stride * u) * 16;
      if (BF16)
        st_bf16x8(a, v[u]);
      else
        st_f32x4(reinterpret_cast<float*>(a), make_float4(__uint_as_float(v[u].x), __uint_as_float(v[u].y),
                                                          __uint_as_float(v[u].z), __uint_as_float(v[u].w)));
    }
  }
  for (; i < v1; i += stride) {
    uint8_t* a = mc + i * 16;
    if (BF16) {
      uint4 v;
      ld_reduce_bf16x8(a, v);
      st_bf16x8(a, v);
    } else {
      float4 f;
      ld_reduce_f32x4(reinterpret_cast<float*>(a), f);
      st_f32x4(reinterpret_cast<float*>(a), f);
    }
  }
}

// One call: a bf16 segment and an fp32 segment of the same multicast buffer, between the
// two cross-rank barriers.
__global__ void __launch_bounds__(kThreads)
    allreduce2_kernel(uint8_t* mc_base, uint32_t* mc_flag, const uint32_t* local_flag, int64_t bf16_off,
                      int64_t bf16_count, int64_t f32_off, int64_t f32_count, int rank, int world,
                      uint32_t epoch) {
  const uint32_t arrivals = static_cast<uint32_t>(world) * gridDim.x;
  if (!barrier(mc_flag, local_flag, arrivals * (2u * epoch + 1u))) return;
  const int cta = static_cast<int>(blockIdx.x), nctas = static_cast<int>(gridDim.x);
  if (bf16_count > 0) reduce_segment<true>(mc_base + bf16_off, bf16_count, rank, world, cta, nctas);
  if (f32_count > 0) reduce_segment<false>(mc_base + f32_off, f32_count, rank, world, cta, nctas);
  barrier(mc_flag, local_flag, arrivals * (2u * epoch + 2u));
}

// ------------------------------------------------------------------ split: switch + peer loads
// The switch's reductions alone leave part of the NVLink bandwidth unused: each rank's link
// carries about one buffer's worth each way in the time the switch takes to reduce it. The split
// call therefore reduces the tail of the bf16 segment without the switch's arithmetic: a rank
// reads its slice of that tail from every rank's copy through plain unicast addresses (its own
// copy from local memory, the others over NVLink), adds the values in fp32 in rank order, rounds
// once to bf16 and broadcasts the sum with multimem.st, as the switch path does. Both parts run
// at once on disjoint CTAs between the same two barriers.
constexpr int kMaxWorld = 8;
constexpr int kPeerUnroll = 2;  // vectors per thread in flight, each read from every rank

struct PeerBases {
  const uint8_t* p[kMaxWorld];  // each rank's copy of the buffer (unicast), ranks 0..world-1
};

// Vectors [vlo, vhi) (16 bytes = 8 bf16 each) of the segment at byte offset `off`: this rank's
// slice of them, over CTAs [0, nctas) of the peer group.
__device__ __forceinline__ void peer_segment(uint8_t* mc, const PeerBases& pb, int64_t off, int64_t vlo,
                                             int64_t vhi, int rank, int world, int cta, int nctas) {
  const int64_t n = vhi - vlo;
  const int64_t per = (n + world - 1) / world;
  const int64_t s0 = vlo + per * rank;
  const int64_t s1 = min(vhi, s0 + per);
  const int64_t stride = static_cast<int64_t>(nctas) * blockDim.x;
  for (int64_t i = s0 + static_cast<int64_t>(cta) * blockDim.x + threadIdx.x; i < s1; i += stride * kPeerUnroll) {
    uint4 x[kPeerUnroll][kMaxWorld];
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t j = i + stride * u;
      if (j < s1) {
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
          if (r < world) x[u][r] = mm::ld_unicast_v4(pb.p[r] + off + j * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < kPeerUnroll; ++u) {
      const int64_t j = i + stride * u;
      if (j >= s1) continue;
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r >= world) continue;
        const uint32_t w[4] = {x[u][r].x, x[u][r].y, x[u][r].z, x[u][r].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // a 32-bit word holds elements 2q (low half) and 2q + 1 (high half)
          acc[2 * q] = __fadd_rn(acc[2 * q], __uint_as_float(w[q] << 16));
          acc[2 * q + 1] = __fadd_rn(acc[2 * q + 1], __uint_as_float(w[q] & 0xffff0000u));
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
        o[q] = *reinterpret_cast<const uint32_t*>(&h);
      }
      st_bf16x8(mc + off + j * 16, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// CTAs [0, gridDim.x - peer_ctas) reduce bf16 elements [0, peer_from) and the fp32 segment in
// the switch; the last peer_ctas CTAs reduce bf16 elements [peer_from, bf16_count) by peer loads.
__global__ void __launch_bounds__(kThreads)
    allreduce_split_kernel(uint8_t* mc_base, PeerBases pb, uint32_t* mc_flag, const uint32_t* local_flag,
                           int64_t bf16_off, int64_t bf16_count, int64_t peer_from, int64_t f32_off,
                           int64_t f32_count, int rank, int world, uint32_t epoch, int peer_ctas) {
  const uint32_t arrivals = static_cast<uint32_t>(world) * gridDim.x;
  if (!barrier(mc_flag, local_flag, arrivals * (2u * epoch + 1u))) return;
  const int switch_ctas = static_cast<int>(gridDim.x) - peer_ctas;
  const int cta = static_cast<int>(blockIdx.x);
  if (cta < switch_ctas) {
    if (peer_from > 0) reduce_segment<true>(mc_base + bf16_off, peer_from, rank, world, cta, switch_ctas);
    if (f32_count > 0) reduce_segment<false>(mc_base + f32_off, f32_count, rank, world, cta, switch_ctas);
  } else if (peer_from < bf16_count) {
    peer_segment(mc_base, pb, bf16_off, peer_from / 8, bf16_count / 8, rank, world, cta - switch_ctas,
                 peer_ctas);
  }
  barrier(mc_flag, local_flag, arrivals * (2u * epoch + 2u));
}

__global__ void __launch_bounds__(kThreads)
    allreduce_kernel(float* mc_data, uint32_t* mc_flag, const uint32_t* local_flag, int64_t lo,
                     int64_t hi, int rank, int world, uint32_t epoch) {
  const uint32_t arrivals = static_cast<uint32_t>(world) * gridDim.x;
  if (!barrier(mc_flag, local_flag, arrivals * (2u * epoch + 1u))) return;
  // slice of [lo, hi) owned by this rank, in float4 units where aligned
  const int64_t n = hi - lo;
  const int64_t per = ((n + world - 1) / world + 3) / 4 * 4;
  const int64_t s0 = lo + per * rank;
  const int64_t s1 = min(hi, s0 + per);
  if (s0 < s1) {
    const int64_t v0 = (s0 + 3) / 4 * 4;
    const int64_t v1 = s1 / 4 * 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (v0 < v1) {
      // kUnroll switch round trips in flight per thread: multimem.ld_reduce has a long
      // latency (the switch gathers from every GPU), so throughput needs many outstanding.
      int64_t i = v0 + 4 * t;
      for (; i + 4 * stride * (kUnroll - 1) < v1; i += 4 * stride * kUnroll) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) ld_reduce_f32x4(mc_data + i + 4 * stride * u, v[u]);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_f32x4(mc_data + i + 4 * stride * u, v[u]);
      }
      for (; i < v1; i += 4 * stride) {
        float4 v;
        ld_reduce_f32x4(mc_data + i, v);
        st_f32x4(mc_data + i, v);
      }
    }
    // unaligned head and tail of the slice
    for (int64_t i = s0 + t; i < min(v0, s1); i += stride) {
      float v;
      ld_reduce_f32(mc_data + i, v);
      st_f32(mc_data + i, v);
    }
    for (int64_t i = max(v1, v0) + t; i < s1; i += stride) {
      float v;
      ld_reduce_f32(mc_data + i, v);
      st_f32(mc_data + i, v);
    }
  }
  barrier(mc_flag, local_flag, arrivals * (2u * epoch + 2u));
}

}  // namespace nvls
}  // namespace c3cu

extern "C" int c3cu_nvls_allreduce(void* mc_base, uint32_t* mc_flag, const uint32_t* local_flag,
                                   int64_t bf16_offset, int64_t bf16_count, int64_t f32_offset,
                                   int64_t f32_count, int rank, int world, uint32_t epoch, int num_ctas,
                                   c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (!mc_base || !mc_flag || !local_flag || bf16_offset < 0 || bf16_count < 0 || f32_offset < 0 ||
      f32_count < 0 || world < 1 || rank < 0 || rank >= world || num_ctas < 1 || num_ctas > 1024) {
    set_error("nvls_allreduce: bad arguments");
    return C3CU_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(mc_base) & 15u) || (bf16_offset & 15) || (f32_offset & 15) ||
      (bf16_count % 8) || (f32_count % 4)) {
    set_error("nvls_allreduce: segments must start on 16 bytes and hold whole 16-byte vectors "
              "(bf16 count %% 8, fp32 count %% 4)");
    return C3CU_ERR_ALIGN;
  }
  return cuda_status(nvls::launch_ar(nvls::allreduce2_kernel, num_ctas, static_cast<cudaStream_t>(stream),
                                     static_cast<uint8_t*>(mc_base), mc_flag, local_flag, bf16_offset, bf16_count,
                                     f32_offset, f32_count, rank, world, epoch),
                     "nvls_allreduce: launch");
}

extern "C" int c3cu_nvls_allreduce_split(void* mc_base, const void* const* peer_bases, uint32_t* mc_flag,
                                         const uint32_t* local_flag, int64_t bf16_offset, int64_t bf16_count,
                                         int64_t bf16_peer_from, int64_t f32_offset, int64_t f32_count, int rank,
                                         int world, uint32_t epoch, int num_ctas, int peer_ctas,
                                         c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (!mc_base || !mc_flag || !local_flag || bf16_offset < 0 || bf16_count < 0 || f32_offset < 0 ||
      f32_count < 0 || world < 1 || world > nvls::kMaxWorld || rank < 0 || rank >= world || num_ctas < 1 ||
      num_ctas > 1024 || bf16_peer_from < 0 || bf16_peer_from > bf16_count || peer_ctas < 0 ||
      peer_ctas > num_ctas) {
    set_error("nvls_allreduce_split: bad arguments (at most 8 ranks; 0 <= bf16_peer_from <= bf16_count; "
              "0 <= peer_ctas <= num_ctas)");
    return C3CU_ERR_INVALID;
  }
  const bool peer_part = bf16_peer_from < bf16_count;
  const bool switch_part = bf16_peer_from > 0 || f32_count > 0;
  if ((peer_part && peer_ctas < 1) || (switch_part && peer_ctas >= num_ctas) || (!peer_part && peer_ctas != 0)) {
    set_error("nvls_allreduce_split: peer_ctas must be >= 1 when bf16_peer_from < bf16_count, 0 when it "
              "equals bf16_count, and leave at least one CTA for the switch part when it is not empty");
    return C3CU_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(mc_base) & 15u) || (bf16_offset & 15) || (f32_offset & 15) ||
      (bf16_count % 8) || (bf16_peer_from % 8) || (f32_count % 4)) {
    set_error("nvls_allreduce_split: segments must start on 16 bytes and hold whole 16-byte vectors "
              "(bf16 count and bf16_peer_from %% 8, fp32 count %% 4)");
    return C3CU_ERR_ALIGN;
  }
  nvls::PeerBases pb{};
  if (peer_part) {
    if (!peer_bases) {
      set_error("nvls_allreduce_split: peer_bases is NULL");
      return C3CU_ERR_INVALID;
    }
    for (int r = 0; r < world; ++r) {
      if (!peer_bases[r] || (reinterpret_cast<uintptr_t>(peer_bases[r]) & 15u)) {
        set_error("nvls_allreduce_split: every rank's base must be a 16-byte-aligned device address");
        return C3CU_ERR_ALIGN;
      }
      pb.p[r] = static_cast<const uint8_t*>(peer_bases[r]);
    }
  }
  return cuda_status(nvls::launch_ar(nvls::allreduce_split_kernel, num_ctas, static_cast<cudaStream_t>(stream),
                                     static_cast<uint8_t*>(mc_base), pb, mc_flag, local_flag, bf16_offset,
                                     bf16_count, bf16_peer_from, f32_offset, f32_count, rank, world, epoch,
                                     peer_ctas),
                     "nvls_allreduce_split: launch");
}

extern "C" int c3cu_nvls_allreduce_f32(float* mc_data, uint32_t* mc_flag, const uint32_t* local_flag,
                                       int64_t lo, int64_t hi, int rank, int world, uint32_t epoch,
                                       int num_ctas, c3cu_stream_t stream) {
  using namespace c3cu;
  int rc = require_sm100();
  if (rc != C3CU_OK) return rc;
  if (!mc_data || !mc_flag || !local_flag || lo < 0 || hi < lo || world < 1 || rank < 0 ||
      rank >= world || num_ctas < 1 || num_ctas > 1024) {
    set_error("nvls_allreduce_f32: bad arguments");
    return C3CU_ERR_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(mc_data) & 15u) != 0u) {
    set_error("nvls_allreduce_f32: multicast base must be 16-byte aligned");
    return C3CU_ERR_ALIGN;
  }
  return cuda_status(nvls::launch_ar(nvls::allreduce_kernel, num_ctas, static_cast<cudaStream_t>(stream), mc_data,
                                     mc_flag, local_flag, lo, hi, rank, world, epoch),
                     "nvls_allreduce_f32: launch");
}

extern "C" int c3cu_set_collective_cluster(int ctas_per_cluster) {
  if (ctas_per_cluster != 1 && ctas_per_cluster != 2) {
    c3cu::set_error("set_collective_cluster: 1 or 2 CTAs per cluster");
    return C3CU_ERR_INVALID;
  }
  c3cu::nvls::g_cluster.store(ctas_per_cluster, std::memory_order_relaxed);
  return C3CU_OK;
}
