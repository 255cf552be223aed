// C-ABI entry points (include/cuopx.h): argument validation, variant
// selection, launch bookkeeping and the device error word.
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {
thread_local const char* t_last_kernel = "none";
// Why the last CUOPX_CUDA_ERROR on this host thread happened (a CUDA error
// name, or a short text for driver-API failures).
thread_local const char* t_last_cuda_error = "none";
std::atomic<int64_t> g_launches{0};
std::atomic<int> g_sm_count[64] = {};

bool overlaps(const void* a, size_t abytes, const void* b, size_t bbytes) {
  if (!a || !b || abytes == 0 || bbytes == 0) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  return a0 < b0 + bbytes && b0 < a0 + abytes;
}

// Bytes spanned by a row-major rows x cols matrix with leading dim ld.
size_t span_bytes(int64_t rows, int64_t cols, int64_t ld, size_t es) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<size_t>((rows - 1) * ld + cols) * es;
}
}  // namespace

// Tracing, off unless asked for: CUOPX_NVTX=1 wraps every compute entry
// point in an NVTX range (visible to Nsight tools), CUOPX_LOG=1 prints one
// line per call (entry point, sizes, kernel launched, status) to stderr.
// Read once; when both are off a call pays one branch.
struct TraceFlags {
  bool nvtx = false, log = false;
  TraceFlags() {
    const char* n = std::getenv("CUOPX_NVTX");
    const char* l = std::getenv("CUOPX_LOG");
    nvtx = n && *n && *n != '0';
    log = l && *l && *l != '0';
  }
};
const TraceFlags& trace_flags() {
  static const TraceFlags f;
  return f;
}

class ApiScope {
 public:
  ApiScope(const char* name, int64_t a, int64_t b, int64_t c, int64_t d = 1) : name_(name) {
    const TraceFlags& f = trace_flags();
    on_ = f.nvtx || f.log;
    if (!on_) return;
    nvtx_ = f.nvtx;
    log_ = f.log;
    dims_[0] = a, dims_[1] = b, dims_[2] = c, dims_[3] = d;
    if (nvtx_) nvtxRangePushA(name);
  }
  int done(int rc) {
    if (on_) {
      if (nvtx_) nvtxRangePop();
      if (log_)
        std::fprintf(stderr, "cuopx: %s %lld x %lld x %lld (x %lld) -> %s, status %d\n", name_,
                     static_cast<long long>(dims_[0]), static_cast<long long>(dims_[1]),
                     static_cast<long long>(dims_[2]), static_cast<long long>(dims_[3]), t_last_kernel, rc);
      on_ = false;
    }
    return rc;
  }
  ~ApiScope() { done(0); }

 private:
  const char* name_;
  bool on_ = false, nvtx_ = false, log_ = false;
  int64_t dims_[4] = {0, 0, 0, 0};
};

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

void note_launch(const char* name) {
  t_last_kernel = name;
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

int check_launch() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CUOPX_SUCCESS : cuda_failure(e);
}

int cuda_failure(cudaError_t e) {
  t_last_cuda_error = cudaGetErrorName(e);
  return CUOPX_CUDA_ERROR;
}

int cuda_failure_text(const char* what) {
  t_last_cuda_error = what;
  return CUOPX_CUDA_ERROR;
}

size_t vector_workspace_size_impl();
int vector_reduce(int op, int64_t n, const float* x, int64_t incx, const float* y, int64_t incy, float* fres,
                  int64_t* ires, void* workspace, size_t ws_bytes, cudaStream_t stream);
int vector_elementwise(int op, int64_t n, float alpha, const float* x, int64_t incx, float* y, int64_t incy,
                       float c, float s, float* xm, cudaStream_t stream);

// Minimum problem size (M*N*K) for the tcgen05 path; below it the SIMT
// kernel finishes before a persistent TMA pipeline has filled.
constexpr double kTcMinWork = 64.0 * 64.0 * 64.0;
// fp32 problems at least this large go to 3xTF32 on the tensor cores
// (unless the FFMA mode is selected).
constexpr double kTf32x3MinWork = 256.0 * 256.0 * 256.0;
std::atomic<int> g_fp32_mode{CUOPX_FP32_AUTO};
int fp32_mode() { return g_fp32_mode.load(std::memory_order_relaxed); }

// Runs variant `v` when it can take `p`; -1 when it cannot (the caller then
// makes the built-in choice).  In a non-default fp32 mode, variants of the
// other fp32 arithmetic are declined: the mode is an accuracy contract.
int run_variant(int v, const GemmProblem& p, cudaStream_t stream) {
  const int mode = g_fp32_mode.load(std::memory_order_relaxed);
  const bool tc_ok = p.K > 0 && gemm_tc_supported(p);
  const bool x3_ok = p.K > 0 && gemm_tf32x3_supported(p) && mode != CUOPX_FP32_FFMA;
  const bool ffma_ok = p.K > 0 && gemm_simt_f32_supported(p) && mode != CUOPX_FP32_TF32X3;
  switch (v) {
    case kVariantTc2: return tc_ok ? gemm_tc2(p, stream, 256) : -1;
    case kVariantTc2x512: return tc_ok ? gemm_tc2(p, stream, 512) : -1;
    case kVariantTc2x128: return tc_ok ? gemm_tc2(p, stream, 128) : -1;
    case kVariantTc128x256: return tc_ok ? gemm_tc(p, stream, 256) : -1;
    case kVariantTc128x128: return tc_ok ? gemm_tc(p, stream, 128) : -1;
    case kVariantTc128x128x2: return tc_ok ? gemm_tc(p, stream, kTc128x128TwoPerSm) : -1;
    case kVariantTc128x64x2: return tc_ok ? gemm_tc(p, stream, kTc128x64TwoPerSm) : -1;
    case kVariantTf32x3_64: return x3_ok ? gemm_tf32x3(p, stream, 64) : -1;
    case kVariantTf32x3_128: return x3_ok ? gemm_tf32x3(p, stream, 128) : -1;
    case kVariantTf32x3_128k2: return x3_ok ? gemm_tf32x3(p, stream, kTf32x3SplitK2) : -1;
    case kVariantTf32x3Pair: return x3_ok ? gemm_tf32x3(p, stream, kTf32x3PairSplitK2) : -1;
    case kVariantFfma: return ffma_ok ? gemm_simt_f32(p, stream) : -1;
    case kVariantGeneric:
      return (p.dtype == CUOPX_F32 && mode == CUOPX_FP32_TF32X3 && gemm_tf32x3_supported(p)) ? -1
                                                                                             : gemm_simt_generic(p, stream);
    default: return -1;
  }
}

int gemm_route(const GemmProblem& p, cudaStream_t stream) {
  const int v = select_gemm_variant(p);  // override or tuning-table row
  if (v != kVariantAuto) {
    const int rc = run_variant(v, p, stream);
    if (rc != -1) return rc;
  }
  const double work = static_cast<double>(p.M) * p.N * p.K * p.batch;
  if (p.K > 0 && work >= kTcMinWork && gemm_tc_supported(p)) return gemm_tc(p, stream);
  const int mode = g_fp32_mode.load(std::memory_order_relaxed);
  if (p.K > 0 && ((mode == CUOPX_FP32_AUTO && work >= kTf32x3MinWork) || mode == CUOPX_FP32_TF32X3) &&
      gemm_tf32x3_supported(p))
    return gemm_tf32x3(p, stream);
  if (p.K > 0 && gemm_simt_f32_supported(p)) return gemm_simt_f32(p, stream);
  return gemm_simt_generic(p, stream);
}

int validate_gemm(const GemmProblem& p) {
  if (dtype_size(p.dtype) == 0) return CUOPX_UNSUPPORTED_TYPE;
  if (p.M < 0 || p.N < 0 || p.K < 0 || p.batch < 0) return CUOPX_INVALID_ARGUMENT;
  if (p.M == 0 || p.N == 0 || p.batch == 0) return CUOPX_SUCCESS;
  const int64_t a_rows = p.transA ? p.K : p.M, a_cols = p.transA ? p.M : p.K;
  const int64_t b_rows = p.transB ? p.N : p.K, b_cols = p.transB ? p.K : p.N;
  if (p.C == nullptr) return CUOPX_INVALID_ARGUMENT;
  if (p.ldc < std::max<int64_t>(1, p.N)) return CUOPX_INVALID_ARGUMENT;
  if (p.K > 0) {
    if (p.A == nullptr || p.B == nullptr) return CUOPX_INVALID_ARGUMENT;
    if (p.lda < std::max<int64_t>(1, a_cols) || p.ldb < std::max<int64_t>(1, b_cols)) return CUOPX_INVALID_ARGUMENT;
  }
  if (p.batch > 1 && (p.strideA < 0 || p.strideB < 0 || p.strideC < 0)) return CUOPX_INVALID_ARGUMENT;
  const size_t es = dtype_size(p.dtype);
  const int64_t nb = p.batch;
  const size_t c_span = span_bytes(p.M, p.N, p.ldc, es) + (nb > 1 ? static_cast<size_t>(p.strideC) * (nb - 1) * es : 0);
  if (p.K > 0) {
    const size_t a_span =
        span_bytes(a_rows, a_cols, p.lda, es) + (nb > 1 ? static_cast<size_t>(p.strideA) * (nb - 1) * es : 0);
    const size_t b_span =
        span_bytes(b_rows, b_cols, p.ldb, es) + (nb > 1 ? static_cast<size_t>(p.strideB) * (nb - 1) * es : 0);
    if (overlaps(p.C, c_span, p.A, a_span) || overlaps(p.C, c_span, p.B, b_span)) return CUOPX_INVALID_ARGUMENT;
  }
  return -1;  // proceed
}

// Argument checks of every GEMV entry point: a status to return, or -1 to
// proceed (M == 0 succeeds with nothing to do).
int validate_gemv(int dtype, int trans, int64_t M, int64_t N, const void* A, int64_t lda, const void* x,
                  const void* y) {
  if (dtype_size(dtype) == 0) return CUOPX_UNSUPPORTED_TYPE;
  if (M < 0 || N < 0) return CUOPX_INVALID_ARGUMENT;
  if (M == 0) return CUOPX_SUCCESS;
  if (y == nullptr) return CUOPX_INVALID_ARGUMENT;
  if (N > 0) {
    if (A == nullptr || x == nullptr) return CUOPX_INVALID_ARGUMENT;
    if (lda < (trans ? M : N)) return CUOPX_INVALID_ARGUMENT;
    const size_t es = dtype_size(dtype);
    const size_t a_span = trans ? span_bytes(N, M, lda, es) : span_bytes(M, N, lda, es);
    if (overlaps(y, M * es, A, a_span) || overlaps(y, M * es, x, N * es)) return CUOPX_INVALID_ARGUMENT;
  }
  return -1;
}

}  // namespace cuopx

using namespace cuopx;

extern "C" {

int cuopx_version(void) { return 100; }

int cuopx_set_fp32_gemm_mode(int mode) {
  if (mode != CUOPX_FP32_AUTO && mode != CUOPX_FP32_FFMA && mode != CUOPX_FP32_TF32X3)
    return CUOPX_INVALID_ARGUMENT;
  g_fp32_mode.store(mode);
  return CUOPX_SUCCESS;
}

int cuopx_get_fp32_gemm_mode(void) { return g_fp32_mode.load(); }

const char* cuopx_last_kernel(void) { return t_last_kernel; }
const char* cuopx_last_cuda_error(void) { return t_last_cuda_error; }

int64_t cuopx_launch_count(void) { return g_launches.load(); }

int cuopx_get_device_error(int* code_out) {
  if (!code_out) return CUOPX_INVALID_ARGUMENT;
  if (cudaDeviceSynchronize() != cudaSuccess) return CUOPX_CUDA_ERROR;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return CUOPX_CUDA_ERROR;
  *code_out = v;
  return CUOPX_SUCCESS;
}

int cuopx_clear_device_error(void) {
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return CUOPX_CUDA_ERROR;
  return CUOPX_SUCCESS;
}

int cuopx_gemm(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha, const void* A,
               int64_t lda, const void* B, int64_t ldb, double beta, void* C, int64_t ldc, void* stream) {
  ApiScope scope("cuopx_gemm", M, N, K);
  GemmProblem p{dtype, transA != 0, transB != 0, M, N, K, alpha, beta, A, lda, 0, B, ldb, 0, C, ldc, 0, 1};
  const int v = validate_gemm(p);
  if (v >= 0) return scope.done(v);
  return scope.done(gemm_route(p, static_cast<cudaStream_t>(stream)));
}

int cuopx_gemm_ex(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha, const void* A,
                  int64_t lda, const void* B, int64_t ldb, double beta, void* C, int64_t ldc, const void* bias,
                  int epilogue, void* stream) {
  ApiScope scope("cuopx_gemm_ex", M, N, K);
  if (epilogue < 0 || epilogue > (CUOPX_EPI_BIAS | CUOPX_EPI_RELU)) return scope.done(CUOPX_INVALID_ARGUMENT);
  if ((epilogue & CUOPX_EPI_BIAS) && bias == nullptr && M > 0 && N > 0) return scope.done(CUOPX_INVALID_ARGUMENT);
  GemmProblem p{dtype, transA != 0, transB != 0, M, N, K, alpha, beta, A, lda, 0, B, ldb, 0, C, ldc, 0, 1};
  p.bias = (epilogue & CUOPX_EPI_BIAS) ? bias : nullptr;
  p.epi = epilogue;
  const int v = validate_gemm(p);
  if (v >= 0) return scope.done(v);
  if (epilogue & CUOPX_EPI_BIAS) {
    const size_t es = dtype_size(dtype);
    if (overlaps(C, span_bytes(M, N, ldc, es), bias, static_cast<size_t>(N) * es))
      return scope.done(CUOPX_INVALID_ARGUMENT);
  }
  return scope.done(gemm_route(p, static_cast<cudaStream_t>(stream)));
}

int cuopx_gemm_strided_batched(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha,
                               const void* A, int64_t lda, int64_t strideA, const void* B, int64_t ldb,
                               int64_t strideB, double beta, void* C, int64_t ldc, int64_t strideC, int64_t batch,
                               void* stream) {
  ApiScope scope("cuopx_gemm_strided_batched", M, N, K, batch);
  GemmProblem p{dtype, transA != 0, transB != 0, M, N, K, alpha, beta, A, lda, strideA, B, ldb, strideB,
                C, ldc, strideC, batch};
  const int v = validate_gemm(p);
  if (v >= 0) return scope.done(v);
  return scope.done(gemm_route(p, static_cast<cudaStream_t>(stream)));
}

size_t cuopx_gemv_workspace_size(int dtype, int trans, int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  return gemv_workspace_size(dtype, trans, M, N);
}

int cuopx_gemv(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A, int64_t lda, const void* x,
               double beta, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  ApiScope scope("cuopx_gemv", M, N, trans);
  const int v = validate_gemv(dtype, trans, M, N, A, lda, x, y);
  if (v >= 0) return scope.done(v);
  return scope.done(gemv_dispatch(dtype, trans, M, N, alpha, A, lda, x, beta, y, workspace, workspace_bytes,
                                  static_cast<cudaStream_t>(stream)));
}

int cuopx_gather_column_blocks(int dtype, int64_t G, int64_t M, int64_t Nb, const void* blocks, void* out,
                               int64_t ldo, void* stream) {
  if (dtype_size(dtype) == 0) return CUOPX_UNSUPPORTED_TYPE;
  if (G < 0 || M < 0 || Nb < 0) return CUOPX_INVALID_ARGUMENT;
  if (G * M * Nb == 0) return CUOPX_SUCCESS;
  if (!blocks || !out || ldo < G * Nb) return CUOPX_INVALID_ARGUMENT;
  return gather_column_blocks(dtype, G, M, Nb, blocks, out, ldo, static_cast<cudaStream_t>(stream));
}

size_t cuopx_vector_workspace_size(int64_t n) {
  (void)n;
  return vector_workspace_size_impl();
}

static int vec_args_ok(int64_t n, const void* x, int64_t incx, const void* y, int64_t incy, bool need_y) {
  if (n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n == 0) return CUOPX_SUCCESS;
  if (!x || incx == 0) return CUOPX_INVALID_ARGUMENT;
  if (need_y && (!y || incy == 0)) return CUOPX_INVALID_ARGUMENT;
  return -1;
}

int cuopx_dot(int64_t n, const float* x, int64_t incx, const float* y, int64_t incy, float* result,
              void* workspace, size_t workspace_bytes, void* stream) {
  if (!result || n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n > 0) {
    const int v = vec_args_ok(n, x, incx, y, incy, true);
    if (v >= 0) return v;
  }
  return vector_reduce(0, n, x, incx, y, incy, result, nullptr, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int cuopx_asum(int64_t n, const float* x, int64_t incx, float* result, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (!result || n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n > 0 && (!x || incx == 0)) return CUOPX_INVALID_ARGUMENT;
  return vector_reduce(1, n, x, incx, nullptr, 1, result, nullptr, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int cuopx_nrm2(int64_t n, const float* x, int64_t incx, float* result, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (!result || n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n > 0 && (!x || incx == 0)) return CUOPX_INVALID_ARGUMENT;
  return vector_reduce(2, n, x, incx, nullptr, 1, result, nullptr, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int cuopx_iamax(int64_t n, const float* x, int64_t incx, int64_t* result, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (!result || n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n > 0 && (!x || incx == 0)) return CUOPX_INVALID_ARGUMENT;
  return vector_reduce(3, n, x, incx, nullptr, 1, nullptr, result, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int cuopx_iamin(int64_t n, const float* x, int64_t incx, int64_t* result, void* workspace, size_t workspace_bytes,
                void* stream) {
  if (!result || n < 0) return CUOPX_INVALID_ARGUMENT;
  if (n > 0 && (!x || incx == 0)) return CUOPX_INVALID_ARGUMENT;
  return vector_reduce(4, n, x, incx, nullptr, 1, nullptr, result, workspace, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

int cuopx_axpy(int64_t n, float alpha, const float* x, int64_t incx, float* y, int64_t incy, void* stream) {
  const int v = vec_args_ok(n, x, incx, y, incy, true);
  if (v >= 0) return v;
  return vector_elementwise(0, n, alpha, x, incx, y, incy, 0.f, 0.f, nullptr, static_cast<cudaStream_t>(stream));
}

int cuopx_scal(int64_t n, float alpha, float* x, int64_t incx, void* stream) {
  const int v = vec_args_ok(n, x, incx, nullptr, 1, false);
  if (v >= 0) return v;
  return vector_elementwise(1, n, alpha, nullptr, incx, nullptr, 1, 0.f, 0.f, x, static_cast<cudaStream_t>(stream));
}

int cuopx_copy(int64_t n, const float* x, int64_t incx, float* y, int64_t incy, void* stream) {
  const int v = vec_args_ok(n, x, incx, y, incy, true);
  if (v >= 0) return v;
  return vector_elementwise(2, n, 0.f, x, incx, y, incy, 0.f, 0.f, nullptr, static_cast<cudaStream_t>(stream));
}

int cuopx_swap(int64_t n, float* x, int64_t incx, float* y, int64_t incy, void* stream) {
  const int v = vec_args_ok(n, x, incx, y, incy, true);
  if (v >= 0) return v;
  return vector_elementwise(3, n, 0.f, nullptr, incx, y, incy, 0.f, 0.f, x, static_cast<cudaStream_t>(stream));
}

int cuopx_rot(int64_t n, float* x, int64_t incx, float* y, int64_t incy, float c, float s, void* stream) {
  const int v = vec_args_ok(n, x, incx, y, incy, true);
  if (v >= 0) return v;
  return vector_elementwise(4, n, 0.f, nullptr, incx, y, incy, c, s, x, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
