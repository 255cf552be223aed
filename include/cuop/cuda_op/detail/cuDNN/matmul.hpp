// MatMul<T>: 2-D C = op(A) op(B) and 3-D batched [B,M,K] x [B,K,N] (reference
// include/cuda_op/detail/cuDNN/matmul.hpp:9-31, src/cuda_op/detail/cuDNN/
// matmul.cu:75-158).  C is resized to the result shape.  The 3-D case is ONE
// strided-batched call (the reference launches one kernel per batch from a
// host loop).  Synchronous like the reference.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class MatMul : public Operator<T> {
 public:
  MatMul(bool transA = false, bool transB = false) : transA_(transA), transB_(transB) {}
  using Operator<T>::Forward;
  StatusCode Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, int batch_dim);
  StatusCode Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) { return Forward(A, B, C, -1); }
  StatusCode Forward(const Tensor<T>&, Tensor<T>&) override { return StatusCode::UNSUPPORTED_TYPE; }

 private:
  bool transA_, transB_;
};

}  // namespace cu_op_mem
