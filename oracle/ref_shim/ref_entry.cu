// C entry points into the reference's own fp32 operators (compiled from the
// reference's sources by oracle/Makefile), used only by the GPU parity tests
// as a second, independent oracle for the fp32 GEMM / GEMV / batched cases.
// Each call goes through the reference's public operator API unchanged:
//   Gemm<float>::SetWeight + Forward   (src/cuda_op/detail/cuBlas/gemm.cu:410-511)
//   Gemv<float>::SetWeight + Forward   (src/cuda_op/detail/cuBlas/gemv.cu:203-256)
//   BatchMatMul<float>::Forward        (src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94)
//   MatMulReluFused<float>::Forward    (src/cuda_op/detail/cuDNN/kernel_fusion.cu:330-370)
// Pointers are device pointers owned by the caller (wrapped in non-owning
// Tensors); the call synchronises before returning.
#include "cuda_op/detail/cuBlas/gemm.hpp"
#include "cuda_op/detail/cuBlas/gemv.hpp"
#include "cuda_op/detail/cuDNN/batchmatmul.hpp"
#include "cuda_op/detail/cuDNN/kernel_fusion.hpp"

using namespace cu_op_mem;

extern "C" int ref_gemm_f32(int transA, int transB, int M, int N, int K, float alpha, const float* A,
                            const float* B, float beta, float* C) {
  Tensor<float> a(const_cast<float*>(A), {static_cast<size_t>(M), static_cast<size_t>(K)});
  Tensor<float> w(const_cast<float*>(B), {static_cast<size_t>(K), static_cast<size_t>(N)});
  Tensor<float> c(C, {static_cast<size_t>(M), static_cast<size_t>(N)});
  int rc;
  {
    Gemm<float> op(transA != 0, transB != 0, alpha, beta);
    op.SetWeight(w);
    rc = static_cast<int>(op.Forward(a, c));
    cudaDeviceSynchronize();
  }
  // Non-owning tensors: drop the pointers so the destructors free nothing.
  new (&a) Tensor<float>();
  new (&w) Tensor<float>();
  new (&c) Tensor<float>();
  return rc;
}

extern "C" int ref_gemv_f32(int transA, int M, int N, float alpha, const float* A, const float* x, float beta,
                            float* y) {
  Tensor<float> a(const_cast<float*>(A), {static_cast<size_t>(M), static_cast<size_t>(N)});
  Tensor<float> xv(const_cast<float*>(x), {static_cast<size_t>(N)});
  Tensor<float> yv(y, {static_cast<size_t>(M)});
  int rc;
  {
    Gemv<float> op(transA != 0, alpha, beta);
    op.SetWeight(xv);
    rc = static_cast<int>(op.Forward(a, yv));
    cudaDeviceSynchronize();
  }
  new (&a) Tensor<float>();
  new (&xv) Tensor<float>();
  new (&yv) Tensor<float>();
  return rc;
}

extern "C" int ref_batchmatmul_f32(int batch, int M, int N, int K, const float* A, const float* B, float* C) {
  Tensor<float> a(const_cast<float*>(A), {static_cast<size_t>(batch), static_cast<size_t>(M), static_cast<size_t>(K)});
  Tensor<float> b(const_cast<float*>(B), {static_cast<size_t>(batch), static_cast<size_t>(K), static_cast<size_t>(N)});
  Tensor<float> c(C, {static_cast<size_t>(batch), static_cast<size_t>(M), static_cast<size_t>(N)});
  int rc;
  {
    BatchMatMul<float> op;
    rc = static_cast<int>(op.Forward(a, b, c, 0));
    cudaDeviceSynchronize();
  }
  new (&a) Tensor<float>();
  new (&b) Tensor<float>();
  new (&c) Tensor<float>();
  return rc;
}

// MatMulReluFused<float>::SetWeight/SetBias + Forward
// (src/cuda_op/detail/cuDNN/kernel_fusion.cu:316-370): C = relu(A*W + bias).
extern "C" int ref_matmul_relu_f32(int transA, int transB, int M, int N, int K, const float* A, const float* W,
                                   const float* bias, float* C) {
  Tensor<float> a(const_cast<float*>(A), {static_cast<size_t>(M), static_cast<size_t>(K)});
  Tensor<float> w(const_cast<float*>(W), {static_cast<size_t>(K), static_cast<size_t>(N)});
  Tensor<float> b(const_cast<float*>(bias), {static_cast<size_t>(N)});
  Tensor<float> c(C, {static_cast<size_t>(M), static_cast<size_t>(N)});
  int rc;
  {
    MatMulReluFused<float> op(transA != 0, transB != 0);
    op.SetWeight(w);
    if (bias) op.SetBias(b);
    std::vector<Tensor<float>*> ins{&a}, outs{&c};
    rc = static_cast<int>(op.Forward(ins, outs));
    cudaDeviceSynchronize();
  }
  new (&a) Tensor<float>();
  new (&w) Tensor<float>();
  new (&b) Tensor<float>();
  new (&c) Tensor<float>();
  return rc;
}
