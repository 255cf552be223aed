// Dot<T>: result = x . y (reference include/cuda_op/detail/cuBlas/dot.hpp,
// src/cuda_op/detail/cuBlas/dot.cu:160-230).  fp32 on the GPU reduction of
// cuopx_dot (deterministic, fixed order); other element types return
// UNSUPPORTED_TYPE.  The result is copied to the host (synchronises).
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Dot : public Operator<T> {
 public:
  Dot() = default;
  StatusCode Forward(const Tensor<T>& x, const Tensor<T>& y, T& result);
  StatusCode Forward(const Tensor<T>&, Tensor<T>&) override { return StatusCode::UNSUPPORTED_TYPE; }
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
