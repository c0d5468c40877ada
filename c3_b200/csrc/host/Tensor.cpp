#include "Tensor.h"

#include <sys/mman.h>

#include <cstdlib>
#include <cstring>

#include "C3/CudaRuntime.h"

namespace {
constexpr size_t kHugeBytes = size_t(2) << 20;
}  // namespace

struct Tensor::Storage {
  void* ptr = nullptr;
  size_t bytes = 0;
  DeviceType device = DeviceType::kCPU;
  bool owned = true;
  // Device memory is stream-ordered on the stream it was allocated on (the allocating
  // thread's current stream) and goes back to the pool on that stream, whichever thread
  // or current stream releases the last reference.
  cudaStream_t stream = nullptr;
  ~Storage() {
    if (!owned || !ptr) return;
    if (device == DeviceType::kCUDA)
      ct::c3::cuda::freeDevice(ptr, stream);
    else
      std::free(ptr);
  }
};

Tensor::Tensor(ShapeTag, const std::vector<size_t>& shape, DType dtype, DeviceType device)
    : shape_(shape), dtype_(dtype), device_(device) {
  auto st = std::make_shared<Storage>();
  st->bytes = numel() * dtypeSize(dtype);
  st->device = device;
  if (device == DeviceType::kCUDA) {
    st->stream = ct::c3::cuda::currentStream();
    st->ptr = ct::c3::cuda::allocDevice(st->bytes);
  } else if (st->bytes >= kHugeBytes) {
    // Large host tensors sit on 2 MiB boundaries and ask for transparent huge pages: a result
    // copied back from the GPU first-touches its pages, and 4 KiB pages would make that a
    // page fault every 4 KiB.
    const size_t rounded = (st->bytes + kHugeBytes - 1) / kHugeBytes * kHugeBytes;
    st->ptr = std::aligned_alloc(kHugeBytes, rounded);
    if (!st->ptr) throw std::bad_alloc();
    madvise(st->ptr, rounded, MADV_HUGEPAGE);  // advisory: ignored where THP is off
  } else {
    const size_t rounded = ((st->bytes + 63) / 64) * 64;
    st->ptr = std::aligned_alloc(64, rounded > 0 ? rounded : 64);
    if (!st->ptr) throw std::bad_alloc();
  }
  storage_ = std::move(st);
}

Tensor Tensor::wrap(void* data, const std::vector<size_t>& shape, DType dtype, DeviceType device) {
  Tensor t;
  t.shape_ = shape;
  t.dtype_ = dtype;
  t.device_ = device;
  auto st = std::make_shared<Storage>();
  st->ptr = data;
  st->bytes = t.numel() * dtypeSize(dtype);
  st->device = device;
  st->owned = false;
  t.storage_ = std::move(st);
  return t;
}

size_t Tensor::numel() const {
  size_t n = 1;
  for (size_t d : shape_) n *= d;
  return n;
}

const void* Tensor::data() const { return storage_ ? storage_->ptr : nullptr; }
void* Tensor::data() { return storage_ ? storage_->ptr : nullptr; }

Tensor Tensor::reshape(const std::vector<size_t>& shape) const {
  size_t n = 1;
  for (size_t d : shape) n *= d;
  if (n != numel()) throw std::runtime_error("reshape: element count mismatch");
  Tensor t = *this;
  t.shape_ = shape;
  return t;
}

Tensor Tensor::to(DeviceType device) const {
  if (!defined()) return Tensor();
  Tensor out(ShapeTag{}, shape_, dtype_, device);
  const size_t bytes = nbytes();
  if (bytes == 0) return out;
  if (device_ == DeviceType::kCPU && device == DeviceType::kCPU) {
    std::memcpy(out.data(), data(), bytes);
    return out;
  }
  cudaStream_t s = ct::c3::cuda::currentStream();
  if (device_ == DeviceType::kCPU) {
    // host -> device through the staging pipeline; `out` is stream-ordered on `s`
    ct::c3::cuda::copyToDevice(out.data(), data(), bytes, s);
    return out;
  }
  if (device == DeviceType::kCPU) {
    ct::c3::cuda::copyToHost(out.data(), data(), bytes, s);
    return out;
  }
  ct::c3::cuda::checkCuda(cudaMemcpyAsync(out.data(), data(), bytes, cudaMemcpyDeviceToDevice, s), "Tensor::to");
  return out;
}
