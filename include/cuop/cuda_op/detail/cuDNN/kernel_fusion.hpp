// Fused operators over the GEMM epilogue (reference
// include/cuda_op/detail/cuDNN/kernel_fusion.hpp:94-111,
// src/cuda_op/detail/cuDNN/kernel_fusion.cu:316-370).
//
// MatMulReluFused<T>: output = relu(input * weight + bias), input [M, K],
// weight [K, N], bias [N] (used when it has N elements, as in the
// reference), output resized to [M, N].  One cuopx_gemm_ex call with the
// bias add and ReLU in the GEMM epilogue (ReLU(x) = x if x > 0 else +0).
// Forward synchronises like the reference; Backward is not provided
// (UNSUPPORTED_OPERATION, as in the reference).  The convolution fusions of
// the reference are not part of this library.
#pragma once

#include <vector>

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class FusedOperator {
 public:
  virtual ~FusedOperator() = default;
  virtual StatusCode Forward(const std::vector<Tensor<T>*>& inputs, std::vector<Tensor<T>*>& outputs) = 0;
  virtual StatusCode Backward(const std::vector<Tensor<T>*>& inputs, const std::vector<Tensor<T>*>& outputs,
                              std::vector<Tensor<T>*>& grad_inputs) = 0;
};

template <typename T>
class MatMulReluFused : public FusedOperator<T> {
 public:
  explicit MatMulReluFused(bool transA = false, bool transB = false) : transA_(transA), transB_(transB) {}

  StatusCode Forward(const std::vector<Tensor<T>*>& inputs, std::vector<Tensor<T>*>& outputs) override;
  StatusCode Backward(const std::vector<Tensor<T>*>&, const std::vector<Tensor<T>*>&,
                      std::vector<Tensor<T>*>&) override {
    return StatusCode::UNSUPPORTED_OPERATION;
  }

  void SetWeight(const Tensor<T>& weight);  // deep copy, as in the reference
  void SetBias(const Tensor<T>& bias);      // deep copy
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  bool transA_, transB_;
  Tensor<T> weight_;
  Tensor<T> bias_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
