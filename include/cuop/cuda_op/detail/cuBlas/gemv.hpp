// Gemv<T>: y = alpha * op(A) * x + beta * y on the B200 kernels.
//
// Interface of the reference's include/cuda_op/detail/cuBlas/gemv.hpp:9-28:
// ctor(transA, alpha, beta), SetWeight(x) deep-copies x, Forward(A, y).
// A has shape [m, n]; x has n entries, y has m.  With transA the buffer is
// read as A[col*m + row] (n rows of m, the reference's gemv.cu:17), i.e.
// y = A_buf^T x.  The split-K scratch comes from the device memory pool,
// grown on demand and kept by the operator.  Goes through cuopx_gemv.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Gemv : public Operator<T> {
 public:
  using Scalar = typename ScalarOf<T>::type;

  explicit Gemv(bool transA = false, Scalar alpha = Scalar(1), Scalar beta = Scalar(0))
      : transA_(transA), alpha_(alpha), beta_(beta) {}
  Gemv(Gemv&&) noexcept = default;
  Gemv& operator=(Gemv&&) noexcept = default;

  StatusCode Forward(const Tensor<T>& input, Tensor<T>& output) override;
  void SetWeight(const Tensor<T>& weight);
  StatusCode operator()(const Tensor<T>& input, Tensor<T>& output) { return Forward(input, output); }

  void SetStream(cudaStream_t s) { stream_ = s; }
  const Tensor<T>& GetWeight() const { return weight_; }
  bool TransA() const { return transA_; }
  Scalar Alpha() const { return alpha_; }
  Scalar Beta() const { return beta_; }

 private:
  bool transA_;
  Scalar alpha_, beta_;
  Tensor<T> weight_;
  Tensor<unsigned char> workspace_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
