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
// No TMA and no multicast TMA loads are used; only multimem loads/stores/reductions.
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
template <bool BF16>
__device__ __forceinline__ void reduce_segment(uint8_t* mc, int64_t count, int rank, int world) {
  constexpr int64_t kPerVec = BF16 ? 8 : 4;
  const int64_t nvec = count / kPerVec;
  const int64_t per = (nvec + world - 1) / world;
  const int64_t v0 = per * rank;
  const int64_t v1 = min(nvec, v0 + per);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = v0 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
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
  if (bf16_count > 0) reduce_segment<true>(mc_base + bf16_off, bf16_count, rank, world);
  if (f32_count > 0) reduce_segment<false>(mc_base + f32_off, f32_count, rank, world);
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
  nvls::allreduce2_kernel<<<num_ctas, nvls::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(mc_base), mc_flag, local_flag, bf16_offset, bf16_count, f32_offset, f32_count,
      rank, world, epoch);
  return cuda_status(cudaGetLastError(), "nvls_allreduce: launch");
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
  nvls::allreduce_kernel<<<num_ctas, nvls::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      mc_data, mc_flag, local_flag, lo, hi, rank, world, epoch);
  return cuda_status(cudaGetLastError(), "nvls_allreduce_f32: launch");
}
