// NVLink multicast (NVLS) primitives shared by the in-switch all-reduce kernels: loads that the
// NVSwitch reduces over every rank's copy, stores that the switch writes into every rank's
// copy, and the release/acquire counters that order them across GPUs.
//
// An address passed as `mc` is a multicast address: every rank bound its copy of the buffer to
// one NVLink multicast object, and an access through the multicast address reaches all copies.
// Besides multimem.* loads, stores and reductions there is one plain 16-byte load through a
// rank's unicast address (ld_unicast_v4); no TMA or bulk copy touches multicast or peer memory.
#pragma once

#include "common.cuh"

namespace c3cu {
namespace mm {

// Sum over all ranks of 8 bf16 values (fp32 accumulation in the switch, one rounding to bf16).
__device__ __forceinline__ void ld_reduce_bf16x8(const void* mc, uint4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
}

__device__ __forceinline__ void st_bf16x8(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void ld_reduce_f32x4(const float* mc, float4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
}

__device__ __forceinline__ void st_f32x4(float* mc, const float4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void ld_reduce_f32(const float* mc, float& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(mc) : "memory");
}

__device__ __forceinline__ void st_f32(float* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

// Adds v to the counter in every rank's copy, after this thread's earlier writes (and what it
// has observed) are visible system-wide.
__device__ __forceinline__ void red_release_add(uint32_t* mc, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// 16 bytes from a rank's own copy of the buffer through its unicast address (this GPU's memory,
// or a peer's over NVLink). Volatile: never served from a line cached by an earlier launch.
__device__ __forceinline__ uint4 ld_unicast_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded acquire-wait until this rank's copy of a monotonic counter reaches `target`
// (wraparound-safe comparison). On time-out records kFaultWaitPeer with `site` and returns false;
// it also gives up at once when this unit's fault word is already set (a peer that missed one
// counter would miss the later ones too, and each would otherwise wait out its own limit).
__device__ __forceinline__ bool wait_counter(const uint32_t* local, uint32_t target, uint64_t limit_ns,
                                             uint32_t site) {
  if (static_cast<int32_t>(ld_acquire_sys(local) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while (static_cast<int32_t>(ld_acquire_sys(local) - target) < 0) {
    if (fault_raised()) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      record_fault(kFaultWaitPeer, site & 0xffffu);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

}  // namespace mm
}  // namespace c3cu
