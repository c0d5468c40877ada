// Host-side helpers shared by the C-ABI translation units: error reporting, device
// properties, and TMA descriptor encoding through the driver entry point (the library
// does not link libcuda directly, so it loads on machines without a GPU driver).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "c3cu.h"

namespace c3cu {

// Records the message returned by c3cu_last_error() for the calling thread.
void set_error(const char* fmt, ...);

// Returns C3CU_ERR_CUDA (and records the message) when `e` is an error.
int cuda_status(cudaError_t e, const char* what);

// Raises the dynamic shared memory limit of `kernel` to `bytes` on the current device, once per
// device: cudaFuncSetAttribute applies to the current device only. `done` is the caller's
// per-kernel bitmask of devices already set (devices 64 and above are set on every call).
int set_max_dynamic_smem(const void* kernel, int bytes, std::atomic<uint64_t>& done, const char* what);

// Multiprocessor count of the current device (cached per device).
int sm_count();

// C3CU_OK when the current device is an sm_100 part; the kernels carry sm_100a code only.
int require_sm100();

// Encodes a 2-D tiled tensor map over a row-major bf16 matrix [rows][cols] with row stride
// `ld` elements, box {box_cols, box_rows} and 128-byte swizzle. Checks the TMA rules
// (16-byte aligned base and stride) before calling the driver.
int encode_bf16_2d_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint32_t box_cols, uint32_t box_rows);

// Called by c3cu_fault_status when a kernel recorded a fault: a split-K GEMM whose adder gave
// up waiting may leave its ticket and ready words non-zero (its partner publishes after the
// adder has reset them), so every pooled split workspace is cleared again on its stream before
// its next launch.
void gemm_invalidate_split_workspaces();

// Whether GEMM and pre-pass kernels are launched with programmatic dependent launch
// (c3cu_set_launch_overlap; off by default).
bool pdl_enabled();

// Launches `kern` on `stream`, with programmatic stream serialization when pdl_enabled().
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u; }

}  // namespace c3cu
