// Minimal tensor of the host framework, with the members C3 uses (shape(), sizes(),
// numel(), device(), dtype(), data_read<T>(), data_write<T>(), reshape(), the
// Tensor(ShapeTag{}, shape, dtype, device) constructor). Storage is shared between views
// and lives either in host memory (kCPU) or in device memory of the current CUDA device
// (kCUDA, stream-ordered allocation). Borrowed memory can be wrapped without ownership.
#pragma once

#include <cstddef>
#include <memory>
#include <stdexcept>
#include <vector>

#include "Ctools.h"

struct ShapeTag {};

class Tensor {
 public:
  Tensor() = default;
  Tensor(ShapeTag, const std::vector<size_t>& shape, DType dtype = DType::kFloat,
         DeviceType device = DeviceType::kCPU);

  // Non-owning view of memory the caller keeps alive (host or device pointer).
  static Tensor wrap(void* data, const std::vector<size_t>& shape, DType dtype, DeviceType device);

  bool defined() const { return storage_ != nullptr; }
  const std::vector<size_t>& shape() const { return shape_; }
  const std::vector<size_t>& sizes() const { return shape_; }
  size_t numel() const;
  size_t nbytes() const { return numel() * dtypeSize(dtype_); }
  DType dtype() const { return dtype_; }
  DeviceType device() const { return device_; }
  bool is_cuda() const { return device_ == DeviceType::kCUDA; }

  const void* data() const;
  void* data();

  // Typed host access (the C3 CPU API); throws for device tensors.
  template <typename T>
  const T* data_read() const {
    if (device_ != DeviceType::kCPU) throw std::runtime_error("data_read on a device tensor");
    return static_cast<const T*>(data());
  }
  template <typename T>
  T* data_write() {
    if (device_ != DeviceType::kCPU) throw std::runtime_error("data_write on a device tensor");
    return static_cast<T*>(data());
  }

  Tensor reshape(const std::vector<size_t>& shape) const;

  // Copy to `device` (host <-> current CUDA device). Device-to-host copies synchronise the
  // current stream so the host data is ready on return.
  Tensor to(DeviceType device) const;

 private:
  struct Storage;
  std::shared_ptr<Storage> storage_;
  std::vector<size_t> shape_;
  DType dtype_ = DType::kFloat;
  DeviceType device_ = DeviceType::kCPU;
};
