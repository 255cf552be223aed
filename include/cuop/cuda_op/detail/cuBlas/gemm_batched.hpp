// GemmBatched<T>: C_b = alpha * op(A_b) * op(B_b) + beta * C_b for every b.
//
// Operator-style front end of the strided-batched path that the reference
// exposes only as a plugin (GemmBatchedJITPlugin, src/jit/Blas/
// gemm_batched_jit_plugin.cu:113-188, setters at :259-283).  Tensors are
// [batch, rows, cols] and contiguous; Forward(A, B, C) checks the shapes
// (C must be allocated, [batch, M, N]).  Goes through
// cuopx_gemm_strided_batched.
#pragma once

#include "cuda_op/abstract/operator.hpp"

namespace cu_op_mem {

template <typename T>
class GemmBatched : public Operator<T> {
 public:
  using Scalar = typename ScalarOf<T>::type;

  GemmBatched(bool transA = false, bool transB = false, Scalar alpha = Scalar(1), Scalar beta = Scalar(0))
      : transA_(transA), transB_(transB), alpha_(alpha), beta_(beta) {}

  StatusCode Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C);
  // Batched GEMM has two operands; the single-input form is not supported.
  StatusCode Forward(const Tensor<T>&, Tensor<T>&) override { return StatusCode::UNSUPPORTED_TYPE; }
  void SetStream(cudaStream_t s) { stream_ = s; }

 private:
  bool transA_, transB_;
  Scalar alpha_, beta_;
  cudaStream_t stream_ = nullptr;
};

}  // namespace cu_op_mem
