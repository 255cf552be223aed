// The dense BLAS plugins and their manager, B200 build.
//
// Class and method names follow the reference (include/jit/Blas/
// gemm_jit_plugin.hpp:13-102, gemm_batched_jit_plugin.hpp:17-122,
// gemv_jit_plugin.hpp:13-106, vector_ops_jit_plugin.hpp:16-154,
// blas_jit_plugins.hpp:24-64).  Every plugin runs the precompiled sm_100a
// kernels through the C ABI (cuopx.h); Compile() validates the configuration
// and marks the plugin ready, Execute() is synchronous and records a
// PerformanceProfile from CUDA events.  BlasJITPluginManager registers every
// name the reference's callers use, including the ones the reference left
// unregistered ("gemm_batched" and its aliases, the vector-op names) and the
// "gemm_jit" key JITWrapper asks for.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "jit/ijit_plugin.hpp"

namespace cu_op_mem {

// Element type of the ExecuteTyped calls below.  The values are the
// CUOPX_F32 / CUOPX_F64 / CUOPX_F16 / CUOPX_BF16 codes of cuopx.h.
enum class DataType { FLOAT32 = 0, FLOAT64 = 1, FLOAT16 = 2, BFLOAT16 = 3 };

// Shared state and bookkeeping of the BLAS plugins.
class BlasPluginBase : public IJITPlugin {
 public:
  StatusCode Initialize() override;
  StatusCode Compile(const JITConfig& config) override;
  void Optimize(const PerformanceProfile& profile) override { last_profile_.optimization_level = profile.optimization_level; }
  void SetConfig(const JITConfig& config) override { config_ = config; }
  JITConfig GetConfig() const override { return config_; }
  void EnableAutoTuning(bool enable) override { auto_tuning_ = enable; }
  bool IsAutoTuningEnabled() const override { return auto_tuning_; }
  PerformanceProfile GetPerformanceProfile() const override { return last_profile_; }
  bool IsInitialized() const override { return initialized_; }
  bool IsCompiled() const override { return compiled_; }
  std::string GetLastError() const override { return last_error_; }
  void Cleanup() override;
  size_t GetMemoryUsage() const override { return memory_usage_; }

  void SetStream(cudaStream_t s) { stream_ = s; }
  size_t GetExecutionCount() const { return executions_; }

 protected:
  // Checks the common Execute preconditions; sets last_error_ on failure.
  StatusCode ready_to_execute();
  // Times `launch` with CUDA events on stream_, synchronises, fills the profile.
  StatusCode timed(const std::function<int()>& launch, double flops, double bytes, std::vector<int> dims);

  JITConfig config_;
  bool initialized_ = false, compiled_ = false, auto_tuning_ = false;
  std::string last_error_;
  PerformanceProfile last_profile_;
  size_t memory_usage_ = 0;
  size_t executions_ = 0;
  cudaStream_t stream_ = nullptr;
};

// C = alpha * op(A) * op(W) + beta * C.  Execute({A}, {C}); W from SetWeight.
class GemmJITPlugin : public BlasPluginBase {
 public:
  StatusCode Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) override;
  std::string GetPluginName() const override { return "gemm_jit"; }
  void SetGemmParams(bool transA, bool transB, float alpha, float beta);
  // Copies W (the reference moved it out of a const reference).
  void SetWeight(const Tensor<float>& weight);
  // Uses W in place; the caller keeps it alive while the plugin runs.
  void BindWeight(const Tensor<float>& weight);
  // The same product for any element type, on raw buffers: the reference's
  // Execute carries only float tensors, so fp16/bf16 operands (fp32
  // accumulation, one rounding of C) come through here.  op(A) is M x K and
  // op(W) is K x N, densely packed row-major buffers of `dtype` (A stored
  // K x M when transA, W stored N x K when transB), C is M x N; transposes
  // and alpha/beta from SetGemmParams, the weight from SetWeight/BindWeight
  // is not used.  Synchronous on the plugin's stream, like Execute.  No
  // counterpart in the reference.
  StatusCode ExecuteTyped(DataType dtype, int64_t M, int64_t N, int64_t K, const void* A, const void* W, void* C);
  static bool SupportsOperator(const std::string& op_name) { return op_name == "gemm" || op_name == "Gemm"; }

 private:
  bool transA_ = false, transB_ = false;
  float alpha_ = 1.f, beta_ = 0.f;
  Tensor<float> weight_;
};

// Strided batched C_b = alpha * op(A_b) op(B_b) + beta * C_b.  Execute({A, B}, {C}).
class GemmBatchedJITPlugin : public BlasPluginBase {
 public:
  StatusCode Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) override;
  std::string GetPluginName() const override { return "gemm_batched_jit"; }
  void SetBatchSize(int batch_size) { batch_ = batch_size; }
  void SetMatrixDimensions(int m, int n, int k) { m_ = m, n_ = n, k_ = k; }
  void SetTransposeOptions(bool transA, bool transB) { transA_ = transA, transB_ = transB; }
  void SetAlphaBeta(float alpha, float beta) { alpha_ = alpha, beta_ = beta; }
  // 0 (the default) means densely packed.
  void SetBatchStride(int strideA, int strideB, int strideC) { sA_ = strideA, sB_ = strideB, sC_ = strideC; }
  // Execute for any element type on raw buffers of `dtype` (fp16/bf16 with
  // fp32 accumulation, which float tensors cannot carry); batch, dimensions,
  // strides, transposes and alpha/beta from the setters.  No counterpart in
  // the reference.
  StatusCode ExecuteTyped(DataType dtype, const void* A, const void* B, void* C);
  static bool SupportsOperator(const std::string& op_name) {
    return op_name == "gemm_batched" || op_name == "GemmBatched" || op_name == "batched_gemm" ||
           op_name == "BatchedGemm";
  }

 private:
  int batch_ = 0, m_ = 0, n_ = 0, k_ = 0;
  bool transA_ = false, transB_ = false;
  float alpha_ = 1.f, beta_ = 0.f;
  int sA_ = 0, sB_ = 0, sC_ = 0;
};

// y = alpha * op(A) x + beta * y.  The plugin's weight is A [M,N];
// Execute({x}, {y}) (roles as in the reference plugin, gemv_jit_plugin.cu:143-153).
class GemvJITPlugin : public BlasPluginBase {
 public:
  StatusCode Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) override;
  std::string GetPluginName() const override { return "gemv_jit"; }
  void SetGemvParams(bool transA, float alpha, float beta);
  void SetWeight(const Tensor<float>& weight);   // copies A
  void BindWeight(const Tensor<float>& weight);  // uses A in place
  // Execute for any element type on raw buffers of `dtype`: y (M) =
  // alpha * op(A) x (N) + beta * y, A densely packed M x N row-major (stored
  // N x M when transA, as the float weight is read); transA and alpha/beta
  // from SetGemvParams, split-K scratch from the plugin's own workspace.
  // The weight from SetWeight/BindWeight is not used.  No counterpart in the
  // reference.
  StatusCode ExecuteTyped(DataType dtype, int64_t M, int64_t N, const void* A, const void* x, void* y);
  void Cleanup() override;
  static bool SupportsOperator(const std::string& op_name) { return op_name == "gemv" || op_name == "Gemv"; }

 private:
  bool transA_ = false;
  float alpha_ = 1.f, beta_ = 0.f;
  Tensor<float> weight_;
  Tensor<unsigned char> workspace_;
};

enum class VectorOpType { DOT, AXPY, SCAL, COPY, SWAP, ROT, NRM2, ASUM, IAMAX, IAMIN };

// Level-1 ops with BLAS semantics.  Execute roles:
//   DOT: {x, y} -> {r[1]};  NRM2/ASUM: {x} -> {r[1]};  IAMAX/IAMIN: {x} -> {r[1]}
//   holding the 1-based index as a float;  AXPY: {x} -> {y} (y += alpha x);
//   SCAL: {x} -> {out} (out = alpha x, in place when out aliases x);
//   COPY: {x} -> {y};  SWAP/ROT: {x} -> {y}, both updated.
class VectorOpsJITPlugin : public BlasPluginBase {
 public:
  StatusCode Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) override;
  std::string GetPluginName() const override { return "vector_ops_jit"; }
  void SetOperationType(VectorOpType op) { op_ = op; }
  VectorOpType GetOperationType() const { return op_; }
  void SetVectorSize(int size) { n_ = size; }
  void SetAlpha(float alpha) { alpha_ = alpha; }
  void SetBeta(float beta) { beta_ = beta; }
  void SetIncrement(int incx, int incy = 1) { incx_ = incx, incy_ = incy; }
  void SetRotationParams(float c, float s) { c_ = c, s_ = s; }
  void Cleanup() override;
  static bool SupportsOperator(const std::string& op_name);
  // "dot"/"Dot" ... -> op type; false for unknown names.
  static bool ParseOperator(const std::string& op_name, VectorOpType* out);

 private:
  VectorOpType op_ = VectorOpType::DOT;
  int n_ = 0;
  float alpha_ = 1.f, beta_ = 0.f, c_ = 1.f, s_ = 0.f;
  int incx_ = 1, incy_ = 1;
  Tensor<unsigned char> workspace_;
};

class BlasJITPluginManager {
 public:
  static BlasJITPluginManager& Instance();
  void RegisterAllPlugins();
  std::vector<std::string> GetSupportedOperators() const;
  bool SupportsOperator(const std::string& op_name) const;
  std::unique_ptr<IJITPlugin> CreatePlugin(const std::string& op_name);

 private:
  BlasJITPluginManager() = default;
  std::unordered_map<std::string, std::function<std::unique_ptr<IJITPlugin>()>> plugin_factories_;
  mutable std::mutex mutex_;
};

inline void RegisterBlasJITPlugins() { BlasJITPluginManager::Instance().RegisterAllPlugins(); }
inline std::vector<std::string> GetSupportedBlasOperators() {
  return BlasJITPluginManager::Instance().GetSupportedOperators();
}
inline bool IsBlasOperatorSupported(const std::string& op) { return BlasJITPluginManager::Instance().SupportsOperator(op); }
inline std::unique_ptr<IJITPlugin> CreateBlasJITPlugin(const std::string& op) {
  return BlasJITPluginManager::Instance().CreatePlugin(op);
}

}  // namespace cu_op_mem
