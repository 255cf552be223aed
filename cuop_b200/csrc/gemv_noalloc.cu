// cuopx_gemv_noalloc: GEMV for callers that must not allocate device memory.
//
// Some hosts cannot call cudaMalloc once they are running: plugin hosts that
// hand out all device memory themselves and forbid allocation after start-up,
// and latency-bound serving loops where an allocation may block on the
// device or fail under memory pressure.  cuopx_gemv needs split-K scratch for
// many shapes, which such callers cannot provide on demand.  This entry point
// runs the same kernels with their scratch in a fixed array that lives in
// this library's device image, so the call itself allocates nothing.
//
// Limits and rules:
//  * kNoAllocScratchBytes (2 MiB) of scratch per device, held by every GPU
//    that loads the library until the process exits.  Calls whose kernel
//    would need more scratch (never more than cuopx_gemv_workspace_size)
//    are rejected with
//    CUOPX_RESOURCE_UNAVAILABLE.  Where the streaming kernels apply (rows
//    16-byte aligned and a multiple of 16 bytes long), the transposed
//    kernel's partials are at most (2 x resident CTAs) strips of 64 16-byte
//    groups, under 1.3 MB for every type at any size; the generic split
//    kernels that take the other shapes can need more (e.g. bf16
//    transposed 8191 x 8192: ~4.8 MB) and such calls are rejected.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * All calls share the one array.  Calls whose kernels overlap on the GPU
//    (different streams, no ordering between them) race on it; serialise them.
//  * The array keeps the previous call's contents; each call clears the
//    split-K arrival counters (the part that must start at zero) with
//    cudaMemsetAsync on the caller's stream before launching.
#include <mutex>

#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;
static_assert(kCounterBytes < kNoAllocScratchBytes, "counter block must fit the scratch");

static __device__ __align__(256) unsigned char g_gemv_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device (looked up once
// per device; the host-side symbol itself is not a device address).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUOPX_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch) != cudaSuccess || p == nullptr) return CUOPX_CUDA_ERROR;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return CUOPX_SUCCESS;
}

// Scratch bytes the kernel that cuopx_gemv will pick for these arguments
// needs: the same planners in the same order as launch_gemv (streaming
// kernels first, then the split-K kernels).
template <typename T>
size_t scratch_for_call(int trans, int64_t M, int64_t N, int64_t lda, const void* A, const void* x) {
  const int sms = device_sm_count();
  const GemvStreamPlan sp = plan_gemv_stream<T>(trans, M, N, lda, A, x, sms);
  if (sp.ok) return (sp.trans && sp.splits > 1) ? kCounterBytes + sp.partial_bytes : 0;
  const GemvPlan gp = plan_gemv<T>(trans, M, N, lda, A, x, sms);
  return gp.splits > 1 ? gp.partial_bytes + gp.counter_bytes : 0;
}

size_t noalloc_need(int dtype, int trans, int64_t M, int64_t N, int64_t lda, const void* A, const void* x) {
  // fp32/fp64 in FFMA mode run gemv_ordered, which needs no scratch.
  if ((dtype == CUOPX_F32 || dtype == CUOPX_F64) && fp32_mode() == CUOPX_FP32_FFMA) return 0;
  switch (dtype) {
    case CUOPX_F32: return scratch_for_call<float>(trans, M, N, lda, A, x);
    case CUOPX_F64: return scratch_for_call<double>(trans, M, N, lda, A, x);
    case CUOPX_F16: return scratch_for_call<__half>(trans, M, N, lda, A, x);
    case CUOPX_BF16: return scratch_for_call<__nv_bfloat16>(trans, M, N, lda, A, x);
    default: return 0;
  }
}

}  // namespace

}  // namespace cuopx

extern "C" int cuopx_gemv_noalloc(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A,
                                  int64_t lda, const void* x, double beta, void* y, void* stream) {
  using namespace cuopx;
  ApiScope scope("cuopx_gemv_noalloc", M, N, trans);
  // The same argument checks as cuopx_gemv, before the scratch is sized.
  const int v = validate_gemv(dtype, trans, M, N, A, lda, x, y);
  if (v >= 0) return scope.done(v);
  const size_t need = N > 0 ? noalloc_need(dtype, trans, M, N, lda, A, x) : 0;
  if (need > kNoAllocScratchBytes) return scope.done(CUOPX_RESOURCE_UNAVAILABLE);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != CUOPX_SUCCESS) return scope.done(rc);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (need > 0 && cudaMemsetAsync(scratch, 0, kCounterBytes, s) != cudaSuccess) return scope.done(CUOPX_CUDA_ERROR);
  return scope.done(gemv_dispatch(dtype, trans, M, N, alpha, A, lda, x, beta, y, scratch, kNoAllocScratchBytes, s));
}
