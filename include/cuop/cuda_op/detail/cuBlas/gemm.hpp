// Gemm<T>: C = alpha * op(A) * op(W) + beta * C on the B200 kernels.
//
// Interface of the reference's include/cuda_op/detail/cuBlas/gemm.hpp:9-59
// (ctor(transA, transB, alpha, beta), SetWeight deep-copies W, Forward(A, C),
// operator(), move-only).  Shapes: A is [M,K] ([K,M] when transA), W is [K,N]
// ([N,K] when transB), C is [M,N]; anything else returns SHAPE_MISMATCH.
// Every kernel honours the transposes (the reference's tiled kernels ignore
// them, gemm.cu:45-292).  T: float, double, __half, __nv_bfloat16 (16-bit
// types accumulate in fp32; alpha/beta are fp32).  Calls are asynchronous on
// the operator's stream (default: the legacy default stream, as in the
// reference) and go through cuopx_gemm.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Gemm : public Operator<T> {
 public:
  using Scalar = typename ScalarOf<T>::type;

  Gemm(bool transA = false, bool transB = false, Scalar alpha = Scalar(1), Scalar beta = Scalar(0))
      : transA_(transA), transB_(transB), alpha_(alpha), beta_(beta) {}
  Gemm(Gemm&&) noexcept = default;
  Gemm& operator=(Gemm&&) noexcept = default;
  Gemm(const Gemm&) = delete;
  Gemm& operator=(const Gemm&) = delete;

  StatusCode Forward(const Tensor<T>& input, Tensor<T>& output) override;
  void SetWeight(const Tensor<T>& weight);
  StatusCode operator()(const Tensor<T>& input, Tensor<T>& output) { return Forward(input, output); }

  void SetStream(cudaStream_t s) { stream_ = s; }
  cudaStream_t GetStream() const { return stream_; }
  const Tensor<T>& GetWeight() const { return weight_; }
  bool TransA() const { return transA_; }
  bool TransB() const { return transB_; }
  Scalar Alpha() const { return alpha_; }
  Scalar Beta() const { return beta_; }

 private:
  bool transA_, transB_;
  Scalar alpha_, beta_;
  Tensor<T> weight_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
