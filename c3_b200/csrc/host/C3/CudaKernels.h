// CompiledKernel implementations bound to the sm_100a kernels of include/c3cu.h. These are
// what C3Engine::compile returns and what the registries install, so a C3 host dispatcher
// reaches the B200 kernels through the unchanged install-and-dispatch API.
//
// Data movement: inputs may live on the host (DeviceType::kCPU, the reference's tensors) or
// on the device (kCUDA). Host inputs are copied to the device, the kernels run on the C3
// stream (CudaRuntime.h), and outputs are returned on the device the inputs came from.
// Arithmetic: bf16 operands use the tcgen05 tensor-core kernels (fp32 accumulation); fp32
// operands use the bit-exact CUDA-core kernels (Precision::kExactF32) or are rounded to
// bf16 first (Precision::kBF16). There is no CPU execution path: failures throw, and the
// registries turn a throw into nullopt as the reference does.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "C3/C3Engine.h"

namespace ct {
namespace c3 {

class CudaKernelBase : public CompiledKernel {
 public:
  CudaKernelBase(std::string key, Precision precision, std::vector<size_t> out_shape)
      : key_(std::move(key)), precision_(precision), out_shape_(std::move(out_shape)) {}
  std::vector<Tensor> execute(const std::vector<Tensor>& inputs) final;
  const std::string& cacheKey() const override { return key_; }
  DeviceType targetDevice() const override { return DeviceType::kCUDA; }
  size_t workspaceBytes() const override { return 0; }
  std::optional<std::vector<size_t>> outShape() const override { return out_shape_; }
  // Short description of the kernel chosen (used in logs and tests).
  virtual std::string describe() const = 0;
  virtual size_t expectedInputs() const = 0;

 protected:
  // Device tensors only; returns device outputs.
  virtual std::vector<Tensor> run(const std::vector<Tensor>& in) = 0;
  std::string key_;
  Precision precision_;
  std::vector<size_t> out_shape_;
};

// MatMul(X, B) + Add(., bias broadcast by index modulo) + ReLU — the region kernel.
// Inputs (positions in the graph's input list): X [M,K], B [K,N] (or [N,K] when trans_b),
// bias [bias_numel]. Outputs: Y [M,N], mask [M, ceil(N/32)] int32 (bit = pre-activation > 0).
class CudaRegionKernel : public CudaKernelBase {
 public:
  CudaRegionKernel(std::string key, Precision p, size_t M, size_t K, size_t N, size_t bias_numel,
                   bool trans_b, std::vector<size_t> input_pos)
      : CudaKernelBase(std::move(key), p, {M, N}), M_(M), K_(K), N_(N), bias_numel_(bias_numel),
        trans_b_(trans_b), pos_(std::move(input_pos)) {}
  std::string describe() const override;
  size_t expectedInputs() const override { return 3; }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  size_t M_, K_, N_, bias_numel_;
  bool trans_b_;
  std::vector<size_t> pos_;  // positions of X, B, bias among the inputs
};

// c3.matmul with transposes folded into the operand reads, optionally followed by an
// elementwise epilogue: out = act(T + bias[idx % bias_numel]) (act: 0 none, 1 ReLU,
// 2 sigmoid, 3 tanh). Inputs: A, B (and bias when has_bias).
class CudaMatMulKernel : public CudaKernelBase {
 public:
  CudaMatMulKernel(std::string key, Precision p, size_t M, size_t K, size_t N, bool trans_a,
                   bool trans_b, bool has_bias, size_t bias_numel, int act,
                   std::vector<size_t> input_pos)
      : CudaKernelBase(std::move(key), p, {M, N}), M_(M), K_(K), N_(N), trans_a_(trans_a),
        trans_b_(trans_b), has_bias_(has_bias), bias_numel_(bias_numel), act_(act),
        pos_(std::move(input_pos)) {}
  std::string describe() const override;
  size_t expectedInputs() const override { return has_bias_ ? 3 : 2; }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  size_t M_, K_, N_;
  bool trans_a_, trans_b_, has_bias_;
  size_t bias_numel_;
  int act_;
  std::vector<size_t> pos_;
};

// ReLU backward Mul(Gt(x, 0), grad). Inputs: grad and x, where x is either the fp32
// pre-activation or the int32 bit mask emitted by CudaRegionKernel.
class CudaReluBackwardKernel : public CudaKernelBase {
 public:
  CudaReluBackwardKernel(std::string key, Precision p, std::vector<size_t> shape,
                         std::vector<size_t> input_pos)
      : CudaKernelBase(std::move(key), p, shape), pos_(std::move(input_pos)) {}
  std::string describe() const override { return "relu_backward"; }
  size_t expectedInputs() const override { return 2; }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  std::vector<size_t> pos_;  // grad, x
};

// SumReduce along axis 0 of a 2-D tensor (the Add-backward bias gradient).
class CudaSumReduceKernel : public CudaKernelBase {
 public:
  CudaSumReduceKernel(std::string key, Precision p, size_t M, size_t N)
      : CudaKernelBase(std::move(key), p, {N}), M_(M), N_(N) {}
  std::string describe() const override { return "sum_reduce_axis0"; }
  size_t expectedInputs() const override { return 1; }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  size_t M_, N_;
};

// Any graph of elementwise nodes (Add/Sub/Mul/Div/Neg/ReLU/Sigmoid/Tanh/Exp/Log/Gt/Const)
// compiled to the register-machine program of c3cu_ew_program, evaluated in one pass.
class CudaElementwiseKernel : public CudaKernelBase {
 public:
  CudaElementwiseKernel(std::string key, Precision p, std::vector<size_t> out_shape,
                        std::vector<uint8_t> code, std::vector<float> constants, int out_reg,
                        size_t n_inputs)
      : CudaKernelBase(std::move(key), p, std::move(out_shape)), code_(std::move(code)),
        consts_(std::move(constants)), out_reg_(out_reg), n_inputs_(n_inputs) {}
  std::string describe() const override;
  size_t expectedInputs() const override { return n_inputs_; }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  std::vector<uint8_t> code_;
  std::vector<float> consts_;
  int out_reg_;
  size_t n_inputs_;
};

// Fused backward of a chain of unary elementwise nodes (the reference's fused backward
// sequences): inputs [grad, x_0, ..., x_{N-1}] (x_k = node k's forward input, k = 0 most
// downstream), outputs the N gradients the nodes pass upstream, from one pass
// (c3cu_ew_backward_chain). node_ops are C3CU_BW_* codes.
class CudaFusedBackwardKernel : public CudaKernelBase {
 public:
  CudaFusedBackwardKernel(std::string key, std::vector<int> node_ops, std::vector<size_t> shape)
      : CudaKernelBase(std::move(key), Precision::kExactF32, std::move(shape)), ops_(std::move(node_ops)) {}
  std::string describe() const override;
  size_t expectedInputs() const override { return 1 + ops_.size(); }

 protected:
  std::vector<Tensor> run(const std::vector<Tensor>& in) override;

 private:
  std::vector<int> ops_;
};

// Lowers a graph (after dead-code elimination) onto one of the kernels above; throws
// std::runtime_error when the graph is outside what the B200 kernels implement.
std::shared_ptr<CudaKernelBase> lowerGraph(const Graph& graph, const CompileOptions& options,
                                           const std::string& key);

}  // namespace c3
}  // namespace ct
