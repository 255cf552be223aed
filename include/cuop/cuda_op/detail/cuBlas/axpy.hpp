// Axpy<T>: y = alpha * x + y (reference include/cuda_op/detail/cuBlas/axpy.hpp,
// src/cuda_op/detail/cuBlas/axpy.cu).  fp32 through cuopx_axpy; other element
// types return UNSUPPORTED_TYPE.  Asynchronous on the operator's stream.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Axpy : public Operator<T> {
 public:
  explicit Axpy(T alpha = T(1)) : alpha_(alpha) {}
  StatusCode Forward(const Tensor<T>& x, Tensor<T>& y) override;
  void SetAlpha(T alpha) { alpha_ = alpha; }
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  T alpha_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
