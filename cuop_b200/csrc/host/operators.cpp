// Operator classes of the C++ facade: each Forward validates shapes the way
// the reference's operators do and makes one call into the C ABI (cuopx.h).
//   Gemm<T>::Forward       reference src/cuda_op/detail/cuBlas/gemm.cu:417-511
//   Gemv<T>::Forward       reference src/cuda_op/detail/cuBlas/gemv.cu:209-256
//   BatchMatMul<T>::Forward reference src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94
//   MatMul<T>::Forward     reference src/cuda_op/detail/cuDNN/matmul.cu:75-158
//   GemmBatched<T>::Forward (plugin semantics, gemm_batched_jit_plugin.cu:113-188)
//   MatMulReluFused<T>::Forward reference src/cuda_op/detail/cuDNN/kernel_fusion.cu:330-370
//   Dot/Axpy/Scal/Copy      reference src/cuda_op/detail/cuBlas/{dot,axpy,scal,copy}.cu
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cuda_op/detail/cuBlas/axpy.hpp"
#include "cuda_op/detail/cuBlas/copy.hpp"
#include "cuda_op/detail/cuBlas/dot.hpp"
#include "cuda_op/detail/cuBlas/gemm.hpp"
#include "cuda_op/detail/cuBlas/gemm_batched.hpp"
#include "cuda_op/detail/cuBlas/gemv.hpp"
#include "cuda_op/detail/cuBlas/scal.hpp"
#include "cuda_op/detail/cuDNN/batchmatmul.hpp"
#include "cuda_op/detail/cuDNN/kernel_fusion.hpp"
#include "cuda_op/detail/cuDNN/matmul.hpp"
#include "cuopx.h"

namespace cu_op_mem {

namespace {

template <typename T> constexpr int dtype_of();
template <> constexpr int dtype_of<float>() { return CUOPX_F32; }
template <> constexpr int dtype_of<double>() { return CUOPX_F64; }
template <> constexpr int dtype_of<__half>() { return CUOPX_F16; }
template <> constexpr int dtype_of<__nv_bfloat16>() { return CUOPX_BF16; }

inline StatusCode to_status(int rc) { return static_cast<StatusCode>(rc); }

template <typename T>
void copy_weight(Tensor<T>& dst, const Tensor<T>& src) {
  dst = Tensor<T>(src.shape());
  if (src.numel()) cudaMemcpy(dst.data(), src.data(), src.bytes(), cudaMemcpyDeviceToDevice);
}

}  // namespace

// ----------------------------------------------------------------- Gemm
template <typename T>
void Gemm<T>::SetWeight(const Tensor<T>& weight) {
  copy_weight(weight_, weight);
}

template <typename T>
StatusCode Gemm<T>::Forward(const Tensor<T>& input, Tensor<T>& output) {
  const auto& as = input.shape();
  const auto& ws = weight_.shape();
  const auto& cs = output.shape();
  if (as.size() != 2 || ws.size() != 2 || cs.size() != 2) return StatusCode::SHAPE_MISMATCH;
  const int64_t M = static_cast<int64_t>(transA_ ? as[1] : as[0]);
  const int64_t K = static_cast<int64_t>(transA_ ? as[0] : as[1]);
  const int64_t Kw = static_cast<int64_t>(transB_ ? ws[1] : ws[0]);
  const int64_t N = static_cast<int64_t>(transB_ ? ws[0] : ws[1]);
  if (Kw != K || static_cast<int64_t>(cs[0]) != M || static_cast<int64_t>(cs[1]) != N)
    return StatusCode::SHAPE_MISMATCH;
  return to_status(cuopx_gemm(dtype_of<T>(), transA_, transB_, M, N, K, static_cast<double>(alpha_),
                              input.data(), static_cast<int64_t>(as[1]), weight_.data(),
                              static_cast<int64_t>(ws[1]), static_cast<double>(beta_), output.data(), N, stream_));
}

// ----------------------------------------------------------------- Gemv
template <typename T>
void Gemv<T>::SetWeight(const Tensor<T>& weight) {
  copy_weight(weight_, weight);
}

template <typename T>
StatusCode Gemv<T>::Forward(const Tensor<T>& input, Tensor<T>& output) {
  if (input.shape().size() != 2) return StatusCode::SHAPE_MISMATCH;
  const int64_t m = static_cast<int64_t>(input.shape()[0]);
  const int64_t n = static_cast<int64_t>(input.shape()[1]);
  if (static_cast<int64_t>(weight_.numel()) != n || static_cast<int64_t>(output.numel()) != m)
    return StatusCode::SHAPE_MISMATCH;
  const size_t need = cuopx_gemv_workspace_size(dtype_of<T>(), transA_, m, n);
  if (need > workspace_.numel()) {
    workspace_ = Tensor<unsigned char>({need});
    workspace_.zero();  // arrival counters start at zero; kernels leave them zeroed
  }
  // Transposed: the [m, n] tensor holds n rows of m (A[col*m + row]).
  const int64_t lda = transA_ ? m : n;
  return to_status(cuopx_gemv(dtype_of<T>(), transA_, m, n, static_cast<double>(alpha_), input.data(), lda,
                              weight_.data(), static_cast<double>(beta_), output.data(), workspace_.data(),
                              workspace_.numel(), stream_));
}

// ----------------------------------------------------------------- GemmBatched
template <typename T>
StatusCode GemmBatched<T>::Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C) {
  const auto &as = A.shape(), &bs = B.shape(), &cs = C.shape();
  if (as.size() != 3 || bs.size() != 3 || cs.size() != 3) return StatusCode::SHAPE_MISMATCH;
  const int64_t batch = static_cast<int64_t>(as[0]);
  const int64_t M = static_cast<int64_t>(transA_ ? as[2] : as[1]);
  const int64_t K = static_cast<int64_t>(transA_ ? as[1] : as[2]);
  const int64_t Kb = static_cast<int64_t>(transB_ ? bs[2] : bs[1]);
  const int64_t N = static_cast<int64_t>(transB_ ? bs[1] : bs[2]);
  if (static_cast<int64_t>(bs[0]) != batch || Kb != K || static_cast<int64_t>(cs[0]) != batch ||
      static_cast<int64_t>(cs[1]) != M || static_cast<int64_t>(cs[2]) != N)
    return StatusCode::SHAPE_MISMATCH;
  return to_status(cuopx_gemm_strided_batched(
      dtype_of<T>(), transA_, transB_, M, N, K, static_cast<double>(alpha_), A.data(),
      static_cast<int64_t>(as[2]), static_cast<int64_t>(as[1] * as[2]), B.data(), static_cast<int64_t>(bs[2]),
      static_cast<int64_t>(bs[1] * bs[2]), static_cast<double>(beta_), C.data(), N, M * N, batch, stream_));
}

// ----------------------------------------------------------------- BatchMatMul
template <typename T>
StatusCode BatchMatMul<T>::Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, int batch_dim) {
  const auto& a = A.shape();
  const auto& b = B.shape();
  if (a.size() < 3 || b.size() < 3 || a.size() != b.size()) return StatusCode::SHAPE_MISMATCH;
  if (batch_dim < 0) batch_dim += static_cast<int>(a.size());
  if (batch_dim < 0 || batch_dim + 2 >= static_cast<int>(a.size())) return StatusCode::SHAPE_MISMATCH;
  int64_t batch = 1;
  for (int i = 0; i <= batch_dim; ++i) {
    if (a[i] != b[i]) return StatusCode::SHAPE_MISMATCH;
    batch *= static_cast<int64_t>(a[i]);
  }
  const int64_t M = static_cast<int64_t>(a[batch_dim + 1]);
  const int64_t K = static_cast<int64_t>(a[batch_dim + 2]);
  const int64_t N = static_cast<int64_t>(b[batch_dim + 2]);
  if (static_cast<int64_t>(b[batch_dim + 1]) != K) return StatusCode::SHAPE_MISMATCH;
  std::vector<std::size_t> c_shape = a;
  c_shape[batch_dim + 2] = static_cast<std::size_t>(N);
  if (C.data() == nullptr || C.shape() != c_shape) C = Tensor<T>(c_shape);
  const int rc = cuopx_gemm_strided_batched(dtype_of<T>(), 0, 0, M, N, K, 1.0, A.data(), K, M * K, B.data(), N,
                                            K * N, 0.0, C.data(), N, M * N, batch, nullptr);
  if (rc != CUOPX_SUCCESS) return to_status(rc);
  return cudaDeviceSynchronize() == cudaSuccess ? StatusCode::SUCCESS : StatusCode::CUDA_ERROR;
}

// ----------------------------------------------------------------- MatMul
template <typename T>
StatusCode MatMul<T>::Forward(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, int batch_dim) {
  (void)batch_dim;  // the reference infers the batch from the ranks, as here
  const auto& a = A.shape();
  const auto& b = B.shape();
  int rc;
  if (a.size() == 2 && b.size() == 2) {
    const int64_t M = static_cast<int64_t>(transA_ ? a[1] : a[0]);
    const int64_t K = static_cast<int64_t>(transA_ ? a[0] : a[1]);
    const int64_t Kb = static_cast<int64_t>(transB_ ? b[1] : b[0]);
    const int64_t N = static_cast<int64_t>(transB_ ? b[0] : b[1]);
    if (K != Kb) return StatusCode::SHAPE_MISMATCH;
    C.resize({static_cast<std::size_t>(M), static_cast<std::size_t>(N)});
    rc = cuopx_gemm(dtype_of<T>(), transA_, transB_, M, N, K, 1.0, A.data(), static_cast<int64_t>(a[1]), B.data(),
                    static_cast<int64_t>(b[1]), 0.0, C.data(), N, nullptr);
  } else if (a.size() == 3 && b.size() == 3) {
    const int64_t batch = static_cast<int64_t>(a[0]);
    const int64_t M = static_cast<int64_t>(transA_ ? a[2] : a[1]);
    const int64_t K = static_cast<int64_t>(transA_ ? a[1] : a[2]);
    const int64_t Kb = static_cast<int64_t>(transB_ ? b[2] : b[1]);
    const int64_t N = static_cast<int64_t>(transB_ ? b[1] : b[2]);
    if (static_cast<int64_t>(b[0]) != batch || K != Kb) return StatusCode::SHAPE_MISMATCH;
    C.resize({static_cast<std::size_t>(batch), static_cast<std::size_t>(M), static_cast<std::size_t>(N)});
    rc = cuopx_gemm_strided_batched(dtype_of<T>(), transA_, transB_, M, N, K, 1.0, A.data(),
                                    static_cast<int64_t>(a[2]), static_cast<int64_t>(a[1] * a[2]), B.data(),
                                    static_cast<int64_t>(b[2]), static_cast<int64_t>(b[1] * b[2]), 0.0, C.data(), N,
                                    M * N, batch, nullptr);
  } else {
    return StatusCode::TENSOR_DIMONSION_MISMATCH;
  }
  if (rc != CUOPX_SUCCESS) return to_status(rc);
  return cudaDeviceSynchronize() == cudaSuccess ? StatusCode::SUCCESS : StatusCode::CUDA_ERROR;
}

// ----------------------------------------------------------------- MatMulReluFused
template <typename T>
void MatMulReluFused<T>::SetWeight(const Tensor<T>& weight) {
  copy_weight(weight_, weight);
}

template <typename T>
void MatMulReluFused<T>::SetBias(const Tensor<T>& bias) {
  copy_weight(bias_, bias);
}

template <typename T>
StatusCode MatMulReluFused<T>::Forward(const std::vector<Tensor<T>*>& inputs, std::vector<Tensor<T>*>& outputs) {
  if (inputs.size() != 1 || outputs.size() != 1 || !inputs[0] || !outputs[0]) return StatusCode::SHAPE_MISMATCH;
  const Tensor<T>& input = *inputs[0];
  Tensor<T>& output = *outputs[0];
  const auto& a = input.shape();
  const auto& w = weight_.shape();
  if (a.size() != 2 || w.size() != 2) return StatusCode::TENSOR_DIMONSION_MISMATCH;
  const int64_t M = static_cast<int64_t>(transA_ ? a[1] : a[0]);
  const int64_t K = static_cast<int64_t>(transA_ ? a[0] : a[1]);
  const int64_t Kw = static_cast<int64_t>(transB_ ? w[1] : w[0]);
  const int64_t N = static_cast<int64_t>(transB_ ? w[0] : w[1]);
  if (Kw != K) return StatusCode::SHAPE_MISMATCH;
  output.resize({static_cast<std::size_t>(M), static_cast<std::size_t>(N)});
  // As in the reference, a bias is used only when it has N elements.
  const bool has_bias = bias_.numel() == static_cast<std::size_t>(N) && N > 0;
  const int epi = CUOPX_EPI_RELU | (has_bias ? CUOPX_EPI_BIAS : 0);
  const int rc = cuopx_gemm_ex(dtype_of<T>(), transA_, transB_, M, N, K, 1.0, input.data(),
                               static_cast<int64_t>(a[1]), weight_.data(), static_cast<int64_t>(w[1]), 0.0,
                               output.data(), N, has_bias ? bias_.data() : nullptr, epi, stream_);
  if (rc != CUOPX_SUCCESS) return to_status(rc);
  return cudaStreamSynchronize(stream_) == cudaSuccess ? StatusCode::SUCCESS : StatusCode::CUDA_ERROR;
}

// ----------------------------------------------------------------- vector operators (fp32)
template <typename T>
StatusCode Dot<T>::Forward(const Tensor<T>& x, const Tensor<T>& y, T& result) {
  if (x.numel() != y.numel()) return StatusCode::SHAPE_MISMATCH;
  if constexpr (!std::is_same<T, float>::value) {
    (void)result;
    return StatusCode::UNSUPPORTED_TYPE;
  } else {
    const int64_t n = static_cast<int64_t>(x.numel());
    const std::size_t ws = cuopx_vector_workspace_size(n);
    Tensor<unsigned char> scratch({ws + 256});
    float* d_result = reinterpret_cast<float*>(scratch.data() + ws);
    // Arrival counters must start at zero (the pool may hand back a used block).
    if (ws && cudaMemsetAsync(scratch.data(), 0, ws, stream_) != cudaSuccess) return StatusCode::CUDA_ERROR;
    const int rc = cuopx_dot(n, x.data(), 1, y.data(), 1, d_result, scratch.data(), ws, stream_);
    if (rc != CUOPX_SUCCESS) return to_status(rc);
    if (cudaMemcpyAsync(&result, d_result, sizeof(float), cudaMemcpyDeviceToHost, stream_) != cudaSuccess ||
        cudaStreamSynchronize(stream_) != cudaSuccess)
      return StatusCode::CUDA_ERROR;
    return StatusCode::SUCCESS;
  }
}

template <typename T>
StatusCode Axpy<T>::Forward(const Tensor<T>& x, Tensor<T>& y) {
  if (x.numel() != y.numel()) return StatusCode::SHAPE_MISMATCH;
  if constexpr (!std::is_same<T, float>::value) {
    return StatusCode::UNSUPPORTED_TYPE;
  } else {
    return to_status(cuopx_axpy(static_cast<int64_t>(x.numel()), alpha_, x.data(), 1, y.data(), 1, stream_));
  }
}

template <typename T>
StatusCode Scal<T>::Forward(Tensor<T>& x) {
  if constexpr (!std::is_same<T, float>::value) {
    return StatusCode::UNSUPPORTED_TYPE;
  } else {
    return to_status(cuopx_scal(static_cast<int64_t>(x.numel()), alpha_, x.data(), 1, stream_));
  }
}

template <typename T>
StatusCode Copy<T>::Forward(const Tensor<T>& input, Tensor<T>& output) {
  if (input.numel() != output.numel()) return StatusCode::SHAPE_MISMATCH;
  if constexpr (!std::is_same<T, float>::value) {
    return StatusCode::UNSUPPORTED_TYPE;
  } else {
    return to_status(cuopx_copy(static_cast<int64_t>(input.numel()), input.data(), 1, output.data(), 1, stream_));
  }
}

template class Dot<float>;
template class Dot<double>;
template class Axpy<float>;
template class Axpy<double>;
template class Scal<float>;
template class Scal<double>;
template class Copy<float>;
template class Copy<double>;

#define CUOP_INSTANTIATE(T)         \
  template class Gemm<T>;           \
  template class Gemv<T>;           \
  template class GemmBatched<T>;    \
  template class BatchMatMul<T>;    \
  template class MatMul<T>;         \
  template class MatMulReluFused<T>;
CUOP_INSTANTIATE(float)
CUOP_INSTANTIATE(double)
CUOP_INSTANTIATE(__half)
CUOP_INSTANTIATE(__nv_bfloat16)
#undef CUOP_INSTANTIATE

}  // namespace cu_op_mem
