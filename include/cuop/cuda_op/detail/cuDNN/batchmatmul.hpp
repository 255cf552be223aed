// BatchMatMul<T>: C[b] = A[b] * B[b] (reference include/cuda_op/detail/cuDNN/
// batchmatmul.hpp:10-18, src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94).
// Leading dims up to batch_dim form the batch; C is (re)allocated when its
// shape differs; one strided-batched call; synchronous like the reference.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class BatchMatMul : public Operator<T> {
 public:
  StatusCode Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, int batch_dim = 0);
  StatusCode Forward(const Tensor<T>&, Tensor<T>&) override { return StatusCode::UNSUPPORTED_TYPE; }
};

}  // namespace cu_op_mem
