// Copy<T>: output = input (reference include/cuda_op/detail/cuBlas/copy.hpp,
// src/cuda_op/detail/cuBlas/copy.cu).  fp32 through cuopx_copy; other element
// types return UNSUPPORTED_TYPE.  Asynchronous on the operator's stream.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class Copy : public Operator<T> {
 public:
  Copy() = default;
  StatusCode Forward(const Tensor<T>& input, Tensor<T>& output) override;
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
