// Library status entry points of the C ABI (include/c3cu.h) and the host helpers of
// host_util.h: per-thread error message, device checks, fault-word folding, and TMA
// descriptor encoding through the driver entry point.
#include <cudaTypedefs.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "host_util.h"

// Fault accessors of the other translation units (each owns one fault word).
int c3cu_fault_get_gemm(uint32_t* out);
int c3cu_fault_clear_gemm();
int c3cu_fault_get_ew(uint32_t* out);
int c3cu_fault_clear_ew();
int c3cu_fault_get_attn(uint32_t* out);
int c3cu_fault_clear_attn();
int c3cu_fault_get_nvls(uint32_t* out);
int c3cu_fault_clear_nvls();
int c3cu_fault_get_train(uint32_t* out);
int c3cu_fault_clear_train();

namespace c3cu {

namespace {
thread_local std::string g_last_error;
}

// Programmatic dependent launch of the GEMM and pre-pass kernels (c3cu_set_launch_overlap).
std::atomic<bool> g_pdl{false};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return C3CU_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return C3CU_ERR_CUDA;
}

int set_max_dynamic_smem(const void* kernel, int bytes, std::atomic<uint64_t>& done, const char* what) {
  int dev = 0;
  int rc = cuda_status(cudaGetDevice(&dev), what);
  if (rc != C3CU_OK) return rc;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t{1} << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return C3CU_OK;
  rc = cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (rc == C3CU_OK && bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
  return rc;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n;
  }
  return cache[dev];
}

int require_sm100() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("no CUDA device: %s", cudaGetErrorString(e));
    return C3CU_ERR_UNSUPPORTED;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    set_error("device %d is sm_%d%d; this library carries sm_100a code only", dev, major, minor);
    return C3CU_ERR_UNSUPPORTED;
  }
  return C3CU_OK;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

int encode_bf16_2d_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint32_t box_cols, uint32_t box_rows) {
  if (!aligned16(base)) {
    set_error("TMA operand base %p is not 16-byte aligned", base);
    return C3CU_ERR_ALIGN;
  }
  if ((ld * 2u) % 16u != 0u || ld < cols) {
    set_error("TMA operand row stride %llu elements (bf16) is not a multiple of 16 bytes or is "
              "smaller than the row length %llu",
              (unsigned long long)ld, (unsigned long long)cols);
    return C3CU_ERR_ALIGN;
  }
  auto fn = get_encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return C3CU_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2u};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d) rows=%llu cols=%llu ld=%llu box=%ux%u",
              (int)r, (unsigned long long)rows, (unsigned long long)cols, (unsigned long long)ld,
              box_cols, box_rows);
    return C3CU_ERR_CUDA;
  }
  return C3CU_OK;
}

}  // namespace c3cu

extern "C" {

int c3cu_version(void) { return 1; }

const char* c3cu_last_error(void) { return c3cu::g_last_error.c_str(); }

int c3cu_set_launch_overlap(int enable) {
  if (enable != 0 && enable != 1) {
    c3cu::set_error("set_launch_overlap: expected 0 or 1, got %d", enable);
    return C3CU_ERR_INVALID;
  }
  c3cu::g_pdl.store(enable != 0, std::memory_order_relaxed);
  return C3CU_OK;
}

int c3cu_device_check(void) { return c3cu::require_sm100(); }

int c3cu_fault_status(uint32_t* code) {
  if (!code) return C3CU_ERR_INVALID;
  *code = 0u;
  int rc = c3cu::cuda_status(cudaDeviceSynchronize(), "c3cu_fault_status: synchronize");
  if (rc != C3CU_OK) return rc;
  uint32_t words[5] = {0u, 0u, 0u, 0u, 0u};
  if (c3cu_fault_get_gemm(&words[0]) || c3cu_fault_get_ew(&words[1]) ||
      c3cu_fault_get_attn(&words[2]) || c3cu_fault_get_nvls(&words[3]) ||
      c3cu_fault_get_train(&words[4])) {
    c3cu::set_error("c3cu_fault_status: reading fault words failed");
    return C3CU_ERR_CUDA;
  }
  for (uint32_t w : words)
    if (w != 0u && *code == 0u) *code = w;
  c3cu_fault_clear_gemm();
  c3cu_fault_clear_ew();
  c3cu_fault_clear_attn();
  c3cu_fault_clear_nvls();
  c3cu_fault_clear_train();
  if (*code != 0u) {
    c3cu::gemm_invalidate_split_workspaces();
    c3cu::set_error("kernel fault recorded: code %u (site %u)", *code & 0xffffu, *code >> 16);
    return C3CU_ERR_FAULT;
  }
  return C3CU_OK;
}

}  // extern "C"
