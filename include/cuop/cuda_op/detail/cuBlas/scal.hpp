// Scal<T>: x = alpha * x (reference include/cuda_op/detail/cuBlas/scal.hpp,
// src/cuda_op/detail/cuBlas/scal.cu).  fp32 through cuopx_scal; other element
// types return UNSUPPORTED_TYPE.  Asynchronous on the operator's stream.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Scal : public Operator<T> {
 public:
  explicit Scal(T alpha = T(1)) : alpha_(alpha) {}
  StatusCode Forward(Tensor<T>& x);
  StatusCode Forward(const Tensor<T>&, Tensor<T>&) override { return StatusCode::UNSUPPORTED_TYPE; }
  void SetAlpha(T alpha) { alpha_ = alpha; }
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  T alpha_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
