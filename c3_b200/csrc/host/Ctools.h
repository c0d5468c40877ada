// Host-framework vocabulary the C3 API is written against. The reference compiles against
// CTorch's Ctools.h, which is not part of the reference tree; this header defines the
// names C3 uses (op, DeviceType, DType) plus kCUDA / kBF16 / kInt32 for the B200 path.
#pragma once

#include <cstddef>
#include <cstdint>

// Operator kinds. The prime codes of the rolling hash are assigned by name
// (C3/RollingHash.cpp), so the numbering here only has to stay below 64 for the
// last-op bitmasks of the registries.
enum class op : uint8_t {
  Add, Sub, Neg, Mul, Div, MatMul, Dot, Cos, Sin, ReLU, Tanh, Sigmoid, GELU, LReLU, Log, Exp,
  Abs, Softmax, Min, Max, MSE, CE, MAE, Conv, Pool, kCount
};

enum class DeviceType : uint8_t { kCPU = 0, kMPS = 1, kDCU = 2, kCUDA = 3 };

enum class DType : uint8_t { kFloat = 0, kBF16 = 1, kInt32 = 2 };

inline size_t dtypeSize(DType t) { return t == DType::kBF16 ? 2u : 4u; }

inline const char* opName(op o) {
  static const char* names[] = {"Add", "Sub", "Neg", "Mul", "Div", "MatMul", "Dot", "Cos", "Sin",
                                "ReLU", "Tanh", "Sigmoid", "GELU", "LReLU", "Log", "Exp", "Abs",
                                "Softmax", "Min", "Max", "MSE", "CE", "MAE", "Conv", "Pool", "kCount"};
  return names[static_cast<size_t>(o)];
}
