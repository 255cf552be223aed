// Plugin layer of the C++ facade: the four BLAS plugins, the registries, the
// global manager and the hardware probe.  Execute() calls the C ABI.
//   GemmJITPlugin::Execute        reference src/jit/Blas/gemm_jit_plugin.cu:147-265
//   GemmBatchedJITPlugin::Execute reference src/jit/Blas/gemm_batched_jit_plugin.cu:113-188
//   GemvJITPlugin::Execute        reference src/jit/Blas/gemv_jit_plugin.cu:126-200
//   VectorOpsJITPlugin::Execute   reference src/jit/Blas/vector_ops_jit_plugin.cu:113-181
//   PluginRegistrar / PluginManager / GlobalJITManager
//                                 reference src/jit/global_jit_manager.cu:14-400
//   BlasJITPluginManager          reference src/jit/Blas/blas_jit_plugin_manager.cu:7-66
//   ExecuteTyped (GEMM, batched GEMM, GEMV plugins): the same calls for
//                                 fp16/bf16/fp64 buffers; no reference
//                                 counterpart (its Execute is float-only)
#include <algorithm>
#include <cctype>
#include <chrono>
#include <fstream>
#include <set>
#include <sstream>

#include "cuopx.h"
#include "jit/Blas/blas_jit_plugins.hpp"
#include "jit/global_jit_manager.hpp"

namespace cu_op_mem {

// ----------------------------------------------------------------- hardware
HardwareSpec QueryHardwareSpec() {
  HardwareSpec hw;
  int dev = 0;
  cudaDeviceProp p;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
    cudaGetLastError();
    return hw;
  }
  hw.compute_capability_major = p.major;
  hw.compute_capability_minor = p.minor;
  hw.num_sms = hw.multi_processor_count = p.multiProcessorCount;
  hw.max_threads_per_sm = p.maxThreadsPerMultiProcessor;
  hw.max_shared_memory_per_sm = static_cast<int>(p.sharedMemPerMultiprocessor);
  hw.max_registers_per_sm = p.regsPerMultiprocessor;
  hw.max_threads_per_block = p.maxThreadsPerBlock;
  hw.max_blocks_per_sm = p.maxBlocksPerMultiProcessor;
  hw.total_global_memory = p.totalGlobalMem;
  hw.memory_bus_width = p.memoryBusWidth;
  int khz = 0;
  if (cudaDeviceGetAttribute(&khz, cudaDevAttrMemoryClockRate, dev) == cudaSuccess) hw.memory_clock_rate = khz / 1000;
  if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, dev) == cudaSuccess) hw.sm_clock_rate = khz / 1000;
  cudaGetLastError();
  hw.supports_tensor_core = p.major >= 7;
  hw.supports_tma = p.major >= 9;
  hw.gpu_name = p.name;
  hw.shared_memory_per_block = static_cast<int>(p.sharedMemPerBlockOptin);
  return hw;
}

// ----------------------------------------------------------------- base
namespace {
// kernel_type values accepted by Compile(): the names the reference's plugins
// used, all served by the built-in variant table, plus the sm_100a families.
const std::set<std::string>& known_kernel_types() {
  static const std::set<std::string> k = {
      "default", "auto", "basic", "tiled", "warp_optimized", "tensor_core", "blocked", "tma", "standard",
      "optimized", "tcgen05", "simt", "stream", "splitk"};
  return k;
}
}  // namespace

StatusCode BlasPluginBase::Initialize() {
  const HardwareSpec hw = QueryHardwareSpec();
  if (hw.compute_capability_major == 0) {
    last_error_ = "no CUDA device";
    return StatusCode::CUDA_DEVICE_ERROR;
  }
  if (hw.compute_capability_major != 10) {
    last_error_ = "libcuopx.so is built for sm_100a (B200); device is sm_" + hw.GetComputeCapabilityString();
    return StatusCode::CUDA_INVALID_DEVICE;
  }
  initialized_ = true;
  last_error_.clear();
  return StatusCode::SUCCESS;
}

StatusCode BlasPluginBase::Compile(const JITConfig& config) {
  if (!initialized_) {
    last_error_ = "plugin not initialized";
    return StatusCode::NOT_INITIALIZED;
  }
  if (!known_kernel_types().count(config.kernel_type)) {
    last_error_ = "unknown kernel_type '" + config.kernel_type + "'";
    return StatusCode::INVALID_CONFIGURATION;
  }
  config_ = config;
  compiled_ = true;
  last_profile_.compilation_time_ms = 0.0;  // ahead-of-time kernels: nothing to compile
  last_profile_.kernel_type = config.kernel_type;
  return StatusCode::SUCCESS;
}

void BlasPluginBase::Cleanup() {
  compiled_ = false;
  memory_usage_ = 0;
}

StatusCode BlasPluginBase::ready_to_execute() {
  if (!compiled_) {
    last_error_ = "plugin not compiled";
    return StatusCode::NOT_COMPILED;
  }
  return StatusCode::SUCCESS;
}

namespace {
// kernel_type as a hint into GEMM variant selection: the reference's SIMT
// variants map to the FFMA kernels (same ascending-k fma chain), everything
// else to the built-in / tuned choice.
const char* variant_hint(const std::string& kernel_type) {
  if (kernel_type == "basic") return "generic";
  if (kernel_type == "tiled" || kernel_type == "warp_optimized" || kernel_type == "blocked" ||
      kernel_type == "simt")
    return "ffma";
  return nullptr;
}
}  // namespace

StatusCode BlasPluginBase::timed(const std::function<int()>& launch, double flops, double bytes,
                                 std::vector<int> dims) {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  const bool ev = cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
  const auto t0 = std::chrono::steady_clock::now();
  if (ev) cudaEventRecord(e0, stream_);
  cuopx_set_gemm_variant_thread(variant_hint(config_.kernel_type));
  const int rc = launch();
  cuopx_set_gemm_variant_thread(nullptr);
  if (ev) cudaEventRecord(e1, stream_);
  const cudaError_t sync = cudaStreamSynchronize(stream_);
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  float ms = 0.f;
  if (ev && rc == CUOPX_SUCCESS && sync == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (rc != CUOPX_SUCCESS) {
    last_error_ = std::string("kernel call failed: ") + StatusCodeToString(static_cast<StatusCode>(rc));
    return static_cast<StatusCode>(rc);
  }
  if (sync != cudaSuccess) {
    last_error_ = cudaGetErrorString(sync);
    return StatusCode::CUDA_ERROR;
  }
  int dev_err = 0;
  if (cuopx_get_device_error(&dev_err) == CUOPX_SUCCESS && dev_err != 0) {
    // A bounded device-side wait gave up: the kernel returned without its result.
    last_error_ = "device-side wait timed out (device error " + std::to_string(dev_err) + ")";
    return StatusCode::EXECUTION_TIMEOUT;
  }
  ++executions_;
  last_profile_.kernel_time_ms = ms;
  last_profile_.execution_time = secs;
  last_profile_.launch_overhead_ms = std::max(0.0, secs * 1e3 - ms);
  last_profile_.gflops = ms > 0 ? flops / (ms * 1e-3) / 1e9 : 0.0;
  last_profile_.throughput = last_profile_.gflops;
  last_profile_.bandwidth_gb_s = ms > 0 ? bytes / (ms * 1e-3) / 1e9 : 0.0;
  last_profile_.kernel_name = cuopx_last_kernel();
  last_profile_.used_tensor_core = last_profile_.kernel_name.rfind("gemm_tc", 0) == 0 ||
                                  last_profile_.kernel_name.rfind("gemm_tf32x3", 0) == 0;
  last_profile_.used_tma = last_profile_.used_tensor_core;
  last_profile_.matrix_size = std::move(dims);
  last_profile_.kernel_type = config_.kernel_type;
  GlobalJITManager::Instance().RecordExecution(secs);
  return StatusCode::SUCCESS;
}

// ----------------------------------------------------------------- GEMM
void GemmJITPlugin::SetGemmParams(bool transA, bool transB, float alpha, float beta) {
  transA_ = transA;
  transB_ = transB;
  alpha_ = alpha;
  beta_ = beta;
}

void GemmJITPlugin::SetWeight(const Tensor<float>& w) {
  weight_ = Tensor<float>(w.shape());
  if (w.numel()) cudaMemcpy(weight_.data(), w.data(), w.bytes(), cudaMemcpyDeviceToDevice);
  memory_usage_ = weight_.bytes();
}

void GemmJITPlugin::BindWeight(const Tensor<float>& w) {
  weight_ = Tensor<float>(w.data(), w.shape());
  memory_usage_ = 0;
}

namespace {
// Bytes per element of a DataType; 0 for a value outside the enum.
size_t typed_size(DataType dt) {
  switch (dt) {
    case DataType::FLOAT32: return 4;
    case DataType::FLOAT64: return 8;
    case DataType::FLOAT16:
    case DataType::BFLOAT16: return 2;
  }
  return 0;
}
}  // namespace

StatusCode GemmJITPlugin::Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  if (inputs.empty() || outputs.empty()) {
    last_error_ = "Execute needs inputs {A} and outputs {C}";
    return StatusCode::INVALID_ARGUMENT;
  }
  const auto& A = inputs[0];
  const auto& as = A.shape();
  const auto& ws = weight_.shape();
  if (as.size() != 2 || ws.size() != 2) {
    last_error_ = "A and W must be 2-D";
    return StatusCode::SHAPE_MISMATCH;
  }
  const int64_t M = static_cast<int64_t>(transA_ ? as[1] : as[0]);
  const int64_t K = static_cast<int64_t>(transA_ ? as[0] : as[1]);
  const int64_t Kw = static_cast<int64_t>(transB_ ? ws[1] : ws[0]);
  const int64_t N = static_cast<int64_t>(transB_ ? ws[0] : ws[1]);
  if (K != Kw) {
    last_error_ = "Matrix dimension mismatch";
    return StatusCode::SHAPE_MISMATCH;
  }
  auto& C = outputs[0];
  if (C.data() == nullptr) C = Tensor<float>({static_cast<size_t>(M), static_cast<size_t>(N)});
  if (C.numel() != static_cast<size_t>(M * N)) {
    last_error_ = "output has the wrong size";
    return StatusCode::SHAPE_MISMATCH;
  }
  const double bytes = 4.0 * (M * K + K * N + M * N * (beta_ != 0.f ? 2 : 1));
  return timed(
      [&] {
        return cuopx_gemm(CUOPX_F32, transA_, transB_, M, N, K, alpha_, A.data(), static_cast<int64_t>(as[1]),
                          weight_.data(), static_cast<int64_t>(ws[1]), beta_, C.data(), N, stream_);
      },
      2.0 * M * N * K, bytes, {static_cast<int>(M), static_cast<int>(N), static_cast<int>(K)});
}

StatusCode GemmJITPlugin::ExecuteTyped(DataType dtype, int64_t M, int64_t N, int64_t K, const void* A,
                                       const void* W, void* C) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  const size_t es = typed_size(dtype);
  if (es == 0) {
    last_error_ = "unsupported element type";
    return StatusCode::UNSUPPORTED_TYPE;
  }
  if (M < 0 || N < 0 || K < 0) {
    last_error_ = "negative matrix dimension";
    return StatusCode::INVALID_ARGUMENT;
  }
  if (M > 0 && N > 0 && (C == nullptr || (K > 0 && (A == nullptr || W == nullptr)))) {
    last_error_ = "ExecuteTyped needs A, W and C buffers";
    return StatusCode::INVALID_ARGUMENT;
  }
  const int64_t lda = std::max<int64_t>(1, transA_ ? M : K), ldb = std::max<int64_t>(1, transB_ ? K : N);
  const double bytes = double(es) * (double(M) * K + double(K) * N + double(M) * N * (beta_ != 0.f ? 2 : 1));
  return timed(
      [&] {
        return cuopx_gemm(static_cast<int>(dtype), transA_, transB_, M, N, K, alpha_, A, lda, W, ldb, beta_, C,
                          std::max<int64_t>(1, N), stream_);
      },
      2.0 * M * N * K, bytes, {static_cast<int>(M), static_cast<int>(N), static_cast<int>(K)});
}

// ----------------------------------------------------------------- batched GEMM
StatusCode GemmBatchedJITPlugin::Execute(const std::vector<Tensor<float>>& inputs,
                                         std::vector<Tensor<float>>& outputs) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  if (inputs.size() < 2 || outputs.empty()) {
    last_error_ = "Execute needs inputs {A, B} and outputs {C}";
    return StatusCode::INVALID_ARGUMENT;
  }
  if (batch_ <= 0 || m_ <= 0 || n_ <= 0 || k_ <= 0) {
    last_error_ = "batch size and matrix dimensions must be set";
    return StatusCode::INVALID_ARGUMENT;
  }
  const int64_t sA = sA_ ? sA_ : int64_t(m_) * k_, sB = sB_ ? sB_ : int64_t(k_) * n_, sC = sC_ ? sC_ : int64_t(m_) * n_;
  const auto &A = inputs[0], &B = inputs[1];
  auto& C = outputs[0];
  if (A.numel() < static_cast<size_t>((batch_ - 1) * sA + int64_t(m_) * k_) ||
      B.numel() < static_cast<size_t>((batch_ - 1) * sB + int64_t(k_) * n_) ||
      C.numel() < static_cast<size_t>((batch_ - 1) * sC + int64_t(m_) * n_)) {
    last_error_ = "tensors smaller than batch x strides";
    return StatusCode::SHAPE_MISMATCH;
  }
  const int64_t lda = transA_ ? m_ : k_, ldb = transB_ ? k_ : n_;
  const double bytes = 4.0 * batch_ * (double(m_) * k_ + double(k_) * n_ + double(m_) * n_);
  return timed(
      [&] {
        return cuopx_gemm_strided_batched(CUOPX_F32, transA_, transB_, m_, n_, k_, alpha_, A.data(), lda, sA,
                                          B.data(), ldb, sB, beta_, C.data(), n_, sC, batch_, stream_);
      },
      2.0 * batch_ * m_ * n_ * double(k_), bytes, {m_, n_, k_});
}

StatusCode GemmBatchedJITPlugin::ExecuteTyped(DataType dtype, const void* A, const void* B, void* C) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  const size_t es = typed_size(dtype);
  if (es == 0) {
    last_error_ = "unsupported element type";
    return StatusCode::UNSUPPORTED_TYPE;
  }
  if (batch_ <= 0 || m_ <= 0 || n_ <= 0 || k_ <= 0) {
    last_error_ = "batch size and matrix dimensions must be set";
    return StatusCode::INVALID_ARGUMENT;
  }
  if (A == nullptr || B == nullptr || C == nullptr) {
    last_error_ = "ExecuteTyped needs A, B and C buffers";
    return StatusCode::INVALID_ARGUMENT;
  }
  const int64_t sA = sA_ ? sA_ : int64_t(m_) * k_, sB = sB_ ? sB_ : int64_t(k_) * n_, sC = sC_ ? sC_ : int64_t(m_) * n_;
  const int64_t lda = transA_ ? m_ : k_, ldb = transB_ ? k_ : n_;
  const double bytes = double(es) * batch_ * (double(m_) * k_ + double(k_) * n_ + double(m_) * n_);
  return timed(
      [&] {
        return cuopx_gemm_strided_batched(static_cast<int>(dtype), transA_, transB_, m_, n_, k_, alpha_, A, lda, sA,
                                          B, ldb, sB, beta_, C, n_, sC, batch_, stream_);
      },
      2.0 * batch_ * m_ * n_ * double(k_), bytes, {m_, n_, k_});
}

// ----------------------------------------------------------------- GEMV
void GemvJITPlugin::SetGemvParams(bool transA, float alpha, float beta) {
  transA_ = transA;
  alpha_ = alpha;
  beta_ = beta;
}

void GemvJITPlugin::SetWeight(const Tensor<float>& w) {
  weight_ = Tensor<float>(w.shape());
  if (w.numel()) cudaMemcpy(weight_.data(), w.data(), w.bytes(), cudaMemcpyDeviceToDevice);
  memory_usage_ = weight_.bytes() + workspace_.bytes();
}

void GemvJITPlugin::BindWeight(const Tensor<float>& w) { weight_ = Tensor<float>(w.data(), w.shape()); }

void GemvJITPlugin::Cleanup() {
  BlasPluginBase::Cleanup();
  workspace_ = Tensor<unsigned char>();
}

StatusCode GemvJITPlugin::Execute(const std::vector<Tensor<float>>& inputs, std::vector<Tensor<float>>& outputs) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  if (inputs.empty() || outputs.empty()) {
    last_error_ = "Execute needs inputs {x} and outputs {y}";
    return StatusCode::INVALID_ARGUMENT;
  }
  if (weight_.shape().size() != 2) {
    last_error_ = "weight (A) must be set and 2-D";
    return StatusCode::SHAPE_MISMATCH;
  }
  const int64_t m = static_cast<int64_t>(weight_.shape()[0]), n = static_cast<int64_t>(weight_.shape()[1]);
  const auto& x = inputs[0];
  auto& y = outputs[0];
  if (static_cast<int64_t>(x.numel()) != n) {
    last_error_ = "Matrix dimension mismatch";
    return StatusCode::SHAPE_MISMATCH;
  }
  if (y.data() == nullptr) y = Tensor<float>({static_cast<size_t>(m)});
  if (static_cast<int64_t>(y.numel()) != m) {
    last_error_ = "output has the wrong size";
    return StatusCode::SHAPE_MISMATCH;
  }
  const size_t need = cuopx_gemv_workspace_size(CUOPX_F32, transA_, m, n);
  if (need > workspace_.numel()) {
    workspace_ = Tensor<unsigned char>({need});
    workspace_.zero();
  }
  memory_usage_ = weight_.bytes() + workspace_.bytes();
  const int64_t lda = transA_ ? m : n;
  return timed(
      [&] {
        return cuopx_gemv(CUOPX_F32, transA_, m, n, alpha_, weight_.data(), lda, x.data(), beta_, y.data(),
                          workspace_.data(), workspace_.numel(), stream_);
      },
      2.0 * m * n, 4.0 * (double(m) * n + n + m), {static_cast<int>(m), static_cast<int>(n), 1});
}

StatusCode GemvJITPlugin::ExecuteTyped(DataType dtype, int64_t M, int64_t N, const void* A, const void* x, void* y) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  const size_t es = typed_size(dtype);
  if (es == 0) {
    last_error_ = "unsupported element type";
    return StatusCode::UNSUPPORTED_TYPE;
  }
  if (M < 0 || N < 0) {
    last_error_ = "negative matrix dimension";
    return StatusCode::INVALID_ARGUMENT;
  }
  if (M > 0 && (y == nullptr || (N > 0 && (A == nullptr || x == nullptr)))) {
    last_error_ = "ExecuteTyped needs A, x and y buffers";
    return StatusCode::INVALID_ARGUMENT;
  }
  const size_t need = cuopx_gemv_workspace_size(static_cast<int>(dtype), transA_, M, N);
  if (need > workspace_.numel()) {
    workspace_ = Tensor<unsigned char>({need});
    workspace_.zero();
  }
  memory_usage_ = weight_.bytes() + workspace_.bytes();
  const int64_t lda = std::max<int64_t>(1, transA_ ? M : N);
  return timed(
      [&] {
        return cuopx_gemv(static_cast<int>(dtype), transA_, M, N, alpha_, A, lda, x, beta_, y, workspace_.data(),
                          workspace_.numel(), stream_);
      },
      2.0 * M * N, double(es) * (double(M) * N + N + M), {static_cast<int>(M), static_cast<int>(N), 1});
}

// ----------------------------------------------------------------- vector ops
bool VectorOpsJITPlugin::ParseOperator(const std::string& name, VectorOpType* out) {
  static const std::pair<const char*, VectorOpType> table[] = {
      {"dot", VectorOpType::DOT},   {"axpy", VectorOpType::AXPY}, {"scal", VectorOpType::SCAL},
      {"copy", VectorOpType::COPY}, {"swap", VectorOpType::SWAP}, {"rot", VectorOpType::ROT},
      {"nrm2", VectorOpType::NRM2}, {"asum", VectorOpType::ASUM}, {"iamax", VectorOpType::IAMAX},
      {"iamin", VectorOpType::IAMIN}};
  for (const auto& e : table) {
    std::string cap = e.first;
    cap[0] = static_cast<char>(std::toupper(cap[0]));
    if (name == e.first || name == cap) {
      if (out) *out = e.second;
      return true;
    }
  }
  return false;
}

bool VectorOpsJITPlugin::SupportsOperator(const std::string& op_name) { return ParseOperator(op_name, nullptr); }

void VectorOpsJITPlugin::Cleanup() {
  BlasPluginBase::Cleanup();
  workspace_ = Tensor<unsigned char>();
}

StatusCode VectorOpsJITPlugin::Execute(const std::vector<Tensor<float>>& inputs,
                                       std::vector<Tensor<float>>& outputs) {
  const StatusCode r = ready_to_execute();
  if (r != StatusCode::SUCCESS) return r;
  if (inputs.empty() || outputs.empty()) {
    last_error_ = "Execute needs at least one input and one output";
    return StatusCode::INVALID_ARGUMENT;
  }
  const auto& x = inputs[0];
  auto& out = outputs[0];
  const int64_t n = n_ > 0 ? n_ : static_cast<int64_t>(x.numel());
  auto span_ok = [&](const Tensor<float>& t, int64_t inc) {
    return n == 0 || static_cast<int64_t>(t.numel()) >= 1 + (n - 1) * (inc < 0 ? -inc : inc);
  };
  if (!span_ok(x, incx_)) {
    last_error_ = "x shorter than n and incx";
    return StatusCode::SHAPE_MISMATCH;
  }
  const bool reduction = op_ == VectorOpType::DOT || op_ == VectorOpType::NRM2 || op_ == VectorOpType::ASUM ||
                         op_ == VectorOpType::IAMAX || op_ == VectorOpType::IAMIN;
  if (reduction && out.data() == nullptr) out = Tensor<float>({1});
  if (!reduction && !span_ok(out, incy_)) {
    last_error_ = "y shorter than n and incy";
    return StatusCode::SHAPE_MISMATCH;
  }
  if (reduction) {
    const size_t need = cuopx_vector_workspace_size(n);
    if (need > workspace_.numel()) {
      workspace_ = Tensor<unsigned char>({need});
      workspace_.zero();
    }
    memory_usage_ = workspace_.bytes();
  }
  void* ws = workspace_.data();
  const size_t wsb = workspace_.numel();
  float* xp = x.data();
  float* yp = out.data();
  switch (op_) {
    case VectorOpType::DOT: {
      if (inputs.size() < 2 || !span_ok(inputs[1], incy_)) {
        last_error_ = "DOT needs inputs {x, y}";
        return StatusCode::INVALID_ARGUMENT;
      }
      float* y2 = inputs[1].data();
      return timed([&] { return cuopx_dot(n, xp, incx_, y2, incy_, yp, ws, wsb, stream_); }, 2.0 * n, 8.0 * n,
                   {static_cast<int>(n), 1, 1});
    }
    case VectorOpType::NRM2:
      return timed([&] { return cuopx_nrm2(n, xp, incx_, yp, ws, wsb, stream_); }, 2.0 * n, 4.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::ASUM:
      return timed([&] { return cuopx_asum(n, xp, incx_, yp, ws, wsb, stream_); }, 1.0 * n, 4.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::IAMAX:
    case VectorOpType::IAMIN: {
      Tensor<int64_t> idx({1});
      const bool mx = op_ == VectorOpType::IAMAX;
      StatusCode s = timed(
          [&] {
            return mx ? cuopx_iamax(n, xp, incx_, idx.data(), ws, wsb, stream_)
                      : cuopx_iamin(n, xp, incx_, idx.data(), ws, wsb, stream_);
          },
          1.0 * n, 4.0 * n, {static_cast<int>(n), 1, 1});
      if (s != StatusCode::SUCCESS) return s;
      int64_t h = 0;
      cudaMemcpy(&h, idx.data(), sizeof(h), cudaMemcpyDeviceToHost);
      const float f = static_cast<float>(h);
      cudaMemcpy(yp, &f, sizeof(f), cudaMemcpyHostToDevice);
      return StatusCode::SUCCESS;
    }
    case VectorOpType::AXPY:
      return timed([&] { return cuopx_axpy(n, alpha_, xp, incx_, yp, incy_, stream_); }, 2.0 * n, 12.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::SCAL:
      if (yp != xp) {
        const int rc = cuopx_copy(n, xp, incx_, yp, incy_, stream_);
        if (rc != CUOPX_SUCCESS) return static_cast<StatusCode>(rc);
      }
      return timed([&] { return cuopx_scal(n, alpha_, yp, yp == xp ? incx_ : incy_, stream_); }, 1.0 * n, 8.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::COPY:
      return timed([&] { return cuopx_copy(n, xp, incx_, yp, incy_, stream_); }, 0.0, 8.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::SWAP:
      return timed([&] { return cuopx_swap(n, xp, incx_, yp, incy_, stream_); }, 0.0, 16.0 * n,
                   {static_cast<int>(n), 1, 1});
    case VectorOpType::ROT:
      return timed([&] { return cuopx_rot(n, xp, incx_, yp, incy_, c_, s_, stream_); }, 6.0 * n, 16.0 * n,
                   {static_cast<int>(n), 1, 1});
  }
  return StatusCode::NOT_IMPLEMENTED;
}

// ----------------------------------------------------------------- registries
PluginRegistrar& PluginRegistrar::Instance() {
  static PluginRegistrar r;
  return r;
}

void PluginRegistrar::RegisterPluginFactory(const std::string& type, std::unique_ptr<IPluginFactory> f) {
  std::lock_guard<std::mutex> lock(mutex_);
  factories_[type] = std::move(f);
}

std::unique_ptr<IJITPlugin> PluginRegistrar::CreatePlugin(const std::string& type) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = factories_.find(type);
  return it == factories_.end() ? nullptr : it->second->CreatePlugin();
}

std::vector<std::string> PluginRegistrar::GetSupportedPluginTypes() const {
  std::lock_guard<std::mutex> lock(mutex_);
  std::vector<std::string> v;
  for (const auto& kv : factories_) v.push_back(kv.first);
  std::sort(v.begin(), v.end());
  return v;
}

bool PluginRegistrar::IsOperatorSupported(const std::string& op) const {
  std::lock_guard<std::mutex> lock(mutex_);
  for (const auto& kv : factories_)
    if (kv.second->SupportsOperator(op)) return true;
  return false;
}

PluginManager& PluginManager::Instance() {
  static PluginManager m;
  return m;
}

void PluginManager::RegisterPlugin(const std::string& name, std::unique_ptr<IJITPlugin> plugin) {
  std::lock_guard<std::mutex> lock(mutex_);
  plugins_[name] = std::move(plugin);
}

IJITPlugin* PluginManager::GetPlugin(const std::string& name) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = plugins_.find(name);
  return it == plugins_.end() ? nullptr : it->second.get();
}

void PluginManager::RemovePlugin(const std::string& name) {
  std::lock_guard<std::mutex> lock(mutex_);
  plugins_.erase(name);
}

void PluginManager::InitializeAllPlugins() {
  std::lock_guard<std::mutex> lock(mutex_);
  for (auto& kv : plugins_) kv.second->Initialize();
}

void PluginManager::CompileAllPlugins(const JITConfig& c) {
  std::lock_guard<std::mutex> lock(mutex_);
  for (auto& kv : plugins_) kv.second->Compile(c);
}

void PluginManager::CleanupAllPlugins() {
  std::lock_guard<std::mutex> lock(mutex_);
  for (auto& kv : plugins_) kv.second->Cleanup();
}

std::vector<std::string> PluginManager::GetActivePlugins() const {
  std::lock_guard<std::mutex> lock(mutex_);
  std::vector<std::string> v;
  for (const auto& kv : plugins_) v.push_back(kv.first);
  std::sort(v.begin(), v.end());
  return v;
}

size_t PluginManager::GetTotalMemoryUsage() const {
  std::lock_guard<std::mutex> lock(mutex_);
  size_t s = 0;
  for (const auto& kv : plugins_) s += kv.second->GetMemoryUsage();
  return s;
}

JITStatistics PluginManager::GetTotalStatistics() const {
  std::lock_guard<std::mutex> lock(mutex_);
  JITStatistics st;
  for (const auto& kv : plugins_) {
    st.active_kernels += kv.second->IsCompiled() ? 1 : 0;
    st.total_compilations += kv.second->IsCompiled() ? 1 : 0;
    st.total_execution_time += kv.second->GetPerformanceProfile().execution_time;
  }
  return st;
}

// ----------------------------------------------------------------- global manager
GlobalJITManager& GlobalJITManager::Instance() {
  static GlobalJITManager m;
  return m;
}

void GlobalJITManager::SetGlobalConfig(const GlobalJITConfig& c) {
  std::lock_guard<std::mutex> lock(mutex_);
  global_config_ = c;
}

GlobalJITConfig GlobalJITManager::GetGlobalConfig() const {
  std::lock_guard<std::mutex> lock(mutex_);
  return global_config_;
}

void GlobalJITManager::SetOperatorConfig(const std::string& op, const JITConfig& c) {
  std::lock_guard<std::mutex> lock(mutex_);
  operator_configs_[op] = c;
}

JITConfig GlobalJITManager::GetOperatorConfig(const std::string& op) const {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = operator_configs_.find(op);
  return it == operator_configs_.end() ? JITConfig() : it->second;
}

StatusCode GlobalJITManager::Initialize() {
  const HardwareSpec hw = QueryHardwareSpec();
  std::lock_guard<std::mutex> lock(mutex_);
  hw_ = hw;
  if (hw.compute_capability_major == 0) return StatusCode::CUDA_DEVICE_ERROR;
  initialized_ = true;
  return StatusCode::SUCCESS;
}

void GlobalJITManager::Cleanup() {
  std::lock_guard<std::mutex> lock(mutex_);
  operator_configs_.clear();
  initialized_ = false;
}

JITStatistics GlobalJITManager::GetStatistics() const {
  std::lock_guard<std::mutex> lock(mutex_);
  return stats_;
}

void GlobalJITManager::ResetStatistics() {
  std::lock_guard<std::mutex> lock(mutex_);
  stats_.Reset();
}

void GlobalJITManager::RecordExecution(double seconds) {
  std::lock_guard<std::mutex> lock(mutex_);
  stats_.total_execution_time += seconds;
}

void GlobalJITManager::ClearAllCaches() {}  // no compiled-code cache exists

// Text format, one operator per line: name kernel_type tile_size num_stages block_size
void GlobalJITManager::SaveCacheToFile(const std::string& path) {
  std::lock_guard<std::mutex> lock(mutex_);
  std::ofstream f(path);
  for (const auto& kv : operator_configs_)
    f << kv.first << ' ' << kv.second.kernel_type << ' ' << kv.second.tile_size << ' ' << kv.second.num_stages
      << ' ' << kv.second.block_size << '\n';
}

void GlobalJITManager::LoadCacheFromFile(const std::string& path) {
  std::ifstream f(path);
  std::string line;
  std::lock_guard<std::mutex> lock(mutex_);
  while (std::getline(f, line)) {
    std::istringstream is(line);
    std::string name;
    JITConfig c;
    if (is >> name >> c.kernel_type >> c.tile_size >> c.num_stages >> c.block_size) operator_configs_[name] = c;
  }
}

// ----------------------------------------------------------------- BLAS manager
BlasJITPluginManager& BlasJITPluginManager::Instance() {
  static BlasJITPluginManager m;
  return m;
}

void BlasJITPluginManager::RegisterAllPlugins() {
  std::lock_guard<std::mutex> lock(mutex_);
  auto gemm = [] { return std::unique_ptr<IJITPlugin>(new GemmJITPlugin()); };
  auto gemv = [] { return std::unique_ptr<IJITPlugin>(new GemvJITPlugin()); };
  auto batched = [] { return std::unique_ptr<IJITPlugin>(new GemmBatchedJITPlugin()); };
  for (const char* n : {"gemm", "Gemm"}) plugin_factories_[n] = gemm;
  for (const char* n : {"gemv", "Gemv"}) plugin_factories_[n] = gemv;
  for (const char* n : {"gemm_batched", "GemmBatched", "batched_gemm", "BatchedGemm"}) plugin_factories_[n] = batched;
  for (const char* n : {"dot", "axpy", "scal", "copy", "swap", "rot", "nrm2", "asum", "iamax", "iamin"}) {
    VectorOpType t;
    VectorOpsJITPlugin::ParseOperator(n, &t);
    auto make = [t] {
      auto p = std::unique_ptr<VectorOpsJITPlugin>(new VectorOpsJITPlugin());
      p->SetOperationType(t);
      return std::unique_ptr<IJITPlugin>(std::move(p));
    };
    std::string cap = n;
    cap[0] = static_cast<char>(std::toupper(cap[0]));
    plugin_factories_[n] = make;
    plugin_factories_[cap] = make;
  }
}

std::vector<std::string> BlasJITPluginManager::GetSupportedOperators() const {
  std::lock_guard<std::mutex> lock(mutex_);
  std::vector<std::string> v;
  for (const auto& kv : plugin_factories_) v.push_back(kv.first);
  std::sort(v.begin(), v.end());
  return v;
}

bool BlasJITPluginManager::SupportsOperator(const std::string& op) const {
  std::lock_guard<std::mutex> lock(mutex_);
  return plugin_factories_.count(op) != 0;
}

std::unique_ptr<IJITPlugin> BlasJITPluginManager::CreatePlugin(const std::string& op) {
  std::lock_guard<std::mutex> lock(mutex_);
  auto it = plugin_factories_.find(op);
  return it == plugin_factories_.end() ? nullptr : it->second();
}

// ----------------------------------------------------------------- static registration
// Registry keys: the reference's factory types ("gemm", "gemv", "gemm_batched",
// "vector_ops") and the plugin names JITWrapper asks for ("*_jit").
CREATE_PLUGIN_FACTORY(GemmJITPlugin);
CREATE_PLUGIN_FACTORY(GemvJITPlugin);
CREATE_PLUGIN_FACTORY(GemmBatchedJITPlugin);
CREATE_PLUGIN_FACTORY(VectorOpsJITPlugin);
REGISTER_JIT_PLUGIN(gemm, GemmJITPlugin);
REGISTER_JIT_PLUGIN(gemm_jit, GemmJITPlugin);
REGISTER_JIT_PLUGIN(gemv, GemvJITPlugin);
REGISTER_JIT_PLUGIN(gemv_jit, GemvJITPlugin);
REGISTER_JIT_PLUGIN(gemm_batched, GemmBatchedJITPlugin);
REGISTER_JIT_PLUGIN(gemm_batched_jit, GemmBatchedJITPlugin);
REGISTER_JIT_PLUGIN(vector_ops, VectorOpsJITPlugin);
REGISTER_JIT_PLUGIN(vector_ops_jit, VectorOpsJITPlugin);

}  // namespace cu_op_mem
