// Internal host-side interfaces between the C-ABI layer (capi.cu) and the
// kernel translation units.  Not installed; the public surface is cuopx.h.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <algorithm>

#include "cuopx.h"

namespace cuopx {

// SM count of the current device (cached per device).
int device_sm_count();

// Record the kernel variant name for cuopx_last_kernel() and bump the
// process-wide launch counter.
void note_launch(const char* name);

// cudaGetLastError -> CUOPX_SUCCESS / CUOPX_CUDA_ERROR.
int check_launch();
// Record why a call fails with CUOPX_CUDA_ERROR (cuopx_last_cuda_error) and
// return CUOPX_CUDA_ERROR.
int cuda_failure(cudaError_t e);
int cuda_failure_text(const char* what);
// Process-wide fp32 arithmetic mode (cuopx_set_fp32_gemm_mode).
int fp32_mode();

// ---- GEMV (gemv.cu) ----
// Argument checks shared by the GEMV entry points (capi.cu): a status, or -1 to proceed.
int validate_gemv(int dtype, int trans, int64_t M, int64_t N, const void* A, int64_t lda, const void* x,
                  const void* y);
size_t gemv_workspace_size(int dtype, int trans, int64_t M, int64_t N);
int gemv_dispatch(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A, int64_t lda,
                  const void* x, double beta, void* y, void* ws, size_t ws_bytes, cudaStream_t stream);

// ---- GEMM problem descriptor shared by all GEMM back-ends ----
struct GemmProblem {
  int dtype;
  bool transA, transB;
  int64_t M, N, K;
  double alpha, beta;
  const void* A;
  int64_t lda, strideA;
  const void* B;
  int64_t ldb, strideB;
  void* C;
  int64_t ldc, strideC;
  int64_t batch;
  // Fused epilogue (cuopx_gemm_ex): CUOPX_EPI_* flags; bias[N] of the
  // problem's dtype when CUOPX_EPI_BIAS is set.
  const void* bias = nullptr;
  int epi = 0;
};

// SIMT back-ends (gemm_simt.cu): generic any-dtype/any-layout kernel and
// the register-blocked fp32 kernel.
int gemm_simt_generic(const GemmProblem& p, cudaStream_t stream);
bool gemm_simt_f32_supported(const GemmProblem& p);
int gemm_simt_f32(const GemmProblem& p, cudaStream_t stream);

// tcgen05/TMA back-end (gemm_tc.cu) for fp16/bf16.
// bn = 0: choose (2-SM kernel for large problems, else BN 256 or 128);
// bn = 128 / 256: the 1-SM kernel with that tile width.
bool gemm_tc_supported(const GemmProblem& p);
// bn = kTc128x128TwoPerSm: 128 x 128 tiles with two CTAs resident per SM.
constexpr int kTc128x128TwoPerSm = -128;
// bn = kTc128x64TwoPerSm: 128 x 64 tiles with two CTAs resident per SM.
constexpr int kTc128x64TwoPerSm = -64;
int gemm_tc(const GemmProblem& p, cudaStream_t stream, int bn = 0);
// The 1-SM kernel (bn 128 or 256) with every output chunk also stored to
// peers[0..npeers) (peer mappings of identically laid out outputs).
int gemm_tc_peers(const GemmProblem& p, void* const* peers, int npeers, cudaStream_t stream, int bn);

// Two-SM (cta_group::2) tcgen05 back-end (gemm_tc2.cu) for large fp16/bf16.
bool gemm_tc2_wanted(const GemmProblem& p);
// pbn: pair tile width, 128, 256 or 512; 0 = choose (gemm_tc2_pick_width).
int gemm_tc2_pick_width(const GemmProblem& p, bool peers);
int gemm_tc2(const GemmProblem& p, cudaStream_t stream, int pbn = 0);
// Same kernel; every output chunk is also stored to peers[0..npeers) (peer
// mappings of identically laid out outputs, offset to this block's columns).
int gemm_tc2_peers(const GemmProblem& p, void* const* peers, int npeers, cudaStream_t stream, int pbn = 0);

// 3xTF32 tcgen05 back-end (gemm_tf32x3.cu) for fp32.
bool gemm_tf32x3_supported(const GemmProblem& p);
int gemm_tf32x3(const GemmProblem& p, cudaStream_t stream, int bn = 0);  // bn: 0 = choose, 64, 128
// bn = kTf32x3SplitK2: 128 x 128 tiles, K split over a pair of CTAs (cluster).
constexpr int kTf32x3SplitK2 = -2;
// bn = kTf32x3PairSplitK2: 256 x 128 tiles on CTA pairs (cta_group::2), K
// split over two pairs (a cluster of four); K-major A only.
constexpr int kTf32x3PairSplitK2 = -3;

// ---- variant selection (host/tuning.cpp) ----
// GEMM variants a tuning table or an override may name.
enum GemmVariant : int {
  kVariantAuto = 0,
  kVariantTc2 = 1,         // 2-SM tcgen05, 256 x 256 pair tiles
  kVariantTc128x256 = 2,   // 1-SM tcgen05
  kVariantTc128x128 = 3,
  kVariantTf32x3_64 = 4,   // 3xTF32, 128 x 64 tiles
  kVariantTf32x3_128 = 5,
  kVariantFfma = 6,        // register-blocked fp32 FFMA
  kVariantGeneric = 7,     // any dtype / layout
  kVariantTc2x512 = 8,     // 2-SM tcgen05, 256 x 512 pair tiles
  kVariantTc128x128x2 = 9, // 1-SM tcgen05, 128 x 128 tiles, two CTAs per SM
  kVariantTc128x64x2 = 10, // 1-SM tcgen05, 128 x 64 tiles, two CTAs per SM
  kVariantTf32x3_128k2 = 11, // 3xTF32, 128 x 128 tiles, K split over a CTA pair
  kVariantTc2x128 = 12,    // 2-SM tcgen05, 256 x 128 pair tiles
  kVariantTf32x3Pair = 13, // 3xTF32, 256 x 128 tiles on CTA pairs, K split over two pairs
  kVariantCount = 14,
};
const char* gemm_variant_name(int v);
// The override (set by cuopx_set_gemm_variant) if any, else the first
// tuning-table row matching the problem, else kVariantAuto.
int select_gemm_variant(const GemmProblem& p);

// Column-block gather (vector_ops.cu).
int gather_column_blocks(int dtype, int64_t G, int64_t M, int64_t Nb, const void* blocks, void* out, int64_t ldo,
                         cudaStream_t stream);

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case CUOPX_F32: return 4;
    case CUOPX_F64: return 8;
    case CUOPX_F16: return 2;
    case CUOPX_BF16: return 2;
    default: return 0;
  }
}

}  // namespace cuopx
