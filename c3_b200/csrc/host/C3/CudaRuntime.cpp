#include "C3/CudaRuntime.h"

#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <vector>

#include "c3cu.h"

namespace ct {
namespace c3 {
namespace cuda {

namespace {
thread_local cudaStream_t t_stream = nullptr;

void configurePool(int dev) {
  static std::mutex mu;
  static std::vector<bool> done;
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, false);
  if (done[dev]) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  done[dev] = true;
}
}  // namespace

cudaStream_t currentStream() { return t_stream; }
void setCurrentStream(cudaStream_t s) { t_stream = s; }

bool deviceAvailable() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

void* allocDevice(size_t bytes) {
  if (bytes == 0) bytes = 256;
  int dev = 0;
  checkCuda(cudaGetDevice(&dev), "allocDevice: cudaGetDevice");
  configurePool(dev);
  void* p = nullptr;
  checkCuda(cudaMallocAsync(&p, bytes, t_stream), "allocDevice: cudaMallocAsync");
  return p;
}

void freeDevice(void* p, cudaStream_t stream) {
  if (p) cudaFreeAsync(p, stream);
}

void checkAbi(int rc, const char* what) {
  if (rc != C3CU_OK) throw std::runtime_error(std::string(what) + ": " + c3cu_last_error());
}

void checkCuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace cuda
}  // namespace c3
}  // namespace ct
