/*
 * oracle/cpu_ref.c — CPU restatement of cuOP's dense BLAS hot-path math.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * cuop_b200/csrc and the timed CPU baseline of bench.py; the product path
 * never links or calls it.
 *
 * The reference (Cyxuan0311/cuOP) has no CPU implementation of GEMM/GEMV;
 * these loops restate the math and the summation order of its CUDA kernels:
 *   - GEMM:    src/cuda_op/detail/cuBlas/gemm.cu:14-42 (gemm_kernel_basic:
 *              sum over k ascending, C = alpha*sum + beta*C, transA reads
 *              A[i*lda+row], transB reads B[col*ldb+i]); the BLOCKED kernel
 *              used at 1024^3 (gemm.cu:249-292) has the same k order.
 *   - GEMV:    src/cuda_op/detail/cuBlas/gemv.cu:10-23 (gemv_kernel; the
 *              transposed form reads A[col*m+row], gemv.cu:17).
 *   - Batched: src/cuda_op/detail/cuDNN/batchmatmul.cu:40-48 (no alpha/beta)
 *              and src/jit/Blas/gemm_batched_jit_plugin.cu:324-330 (with
 *              alpha/beta, strides strideA/B/C).
 * Every output is one fused multiply-add chain over k in ascending order
 * (nvcc contracts `sum += a*b` into FFMA), then the epilogue
 * `alpha * sum + beta * C` (gemm.cu:41, gemv.cu:21) the way nvcc builds it:
 * r = fma(alpha, sum, round(beta*c)) when beta != 0, else round(alpha*sum)
 * (C is not read).  That form was pinned by running the reference's own
 * kernels on a B200 with alpha = 0.7, beta = 1.3: it matched every output
 * bit, while rounding alpha*sum separately, or fma(beta, c, alpha*sum), did
 * not (tests/test_reference_bitexact_gpu.py keeps that check).  fp16/bf16
 * inputs are widened to fp32 exactly, accumulated in fp32, and the result
 * rounded once to nearest-even.
 *
 * Build: oracle/Makefile (gcc -O3 -march=x86-64-v3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API __attribute__((visibility("default")))

/* The reference's epilogue alpha*sum + beta*c (see the header comment). */
static inline float axpby_f32(float alpha, float sum, float beta, float c) {
  return beta != 0.0f ? fmaf(alpha, sum, beta * c) : alpha * sum;
}

/* ------------------------------------------------------------------ RNG --
 * Counter-based splitmix64: element i of a tensor with seed s is
 * mix(s + (i+1) * golden); independent of thread count.                  */
static inline uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

/* uniform[lo, hi): u = (z >> 40) * 2^-24, value = lo + (hi - lo) * u. */
ORACLE_API void oracle_fill_uniform_f32(float* out, int64_t n, uint64_t seed, float lo, float hi) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float u = (float)(splitmix64_at(seed, (uint64_t)i) >> 40) * (1.0f / 16777216.0f);
    out[i] = lo + (hi - lo) * u;
  }
}

/* N(mean, std): Box-Muller in fp64 on pairs (2p, 2p+1). */
ORACLE_API void oracle_fill_normal_f32(float* out, int64_t n, uint64_t seed, double mean, double stddev) {
  const int64_t pairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (int64_t p = 0; p < pairs; ++p) {
    const double u1 = ((double)(splitmix64_at(seed, (uint64_t)(2 * p)) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(splitmix64_at(seed, (uint64_t)(2 * p + 1)) >> 11) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1));
    const double a = 6.283185307179586476925286766559 * u2;
    out[2 * p] = (float)(mean + stddev * r * cos(a));
    if (2 * p + 1 < n) out[2 * p + 1] = (float)(mean + stddev * r * sin(a));
  }
}

/* ------------------------------------------------------------- rounding --
 * Round-to-nearest-even conversions written from the IEEE 754 binary16 and
 * bfloat16 bit layouts.                                                    */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline uint16_t f32_to_bf16(float f) {
  const uint32_t x = f2u(f);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x0040u); /* quiet NaN */
  return (uint16_t)((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}
static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

static inline uint16_t f32_to_f16(float f) {
  const uint32_t x = f2u(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x0200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 -> inf */
  if (ax < 0x38800000u) {                                     /* below 2^-14: subnormal or zero */
    if (ax < 0x33000000u) return (uint16_t)sign;               /* below 2^-25 */
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const int shift = 126 - (int)e; /* 14..24 */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  const uint32_t r = ax - 0x38000000u; /* rebias 127 -> 15 */
  uint32_t q = r >> 13;
  const uint32_t rem = r & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;
  return (uint16_t)(sign | q);
}
static inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  if (e == 0) {
    if (m == 0) return u2f(sign);
    const float v = (float)m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
    return sign ? -v : v;
  }
  if (e == 31) return u2f(sign | 0x7F800000u | (m << 13));
  return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* dtype codes match include/cuopx.h: 2 = f16, 3 = bf16 */
static inline float lowp_to_f32(int dtype, uint16_t h) { return dtype == 3 ? bf16_to_f32(h) : f16_to_f32(h); }
static inline uint16_t f32_to_lowp(int dtype, float f) { return dtype == 3 ? f32_to_bf16(f) : f32_to_f16(f); }

ORACLE_API void oracle_f32_to_lowp(int dtype, const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_lowp(dtype, in[i]);
}
ORACLE_API void oracle_lowp_to_f32(int dtype, const uint16_t* in, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = lowp_to_f32(dtype, in[i]);
}

/* --------------------------------------------------------------- GEMM --
 * Row-major; op(A) is M x K, op(B) is K x N.  Loop order i, k, j keeps
 * each output's fma chain in ascending k while vectorising over j.        */
static inline float a_at_f32(const float* A, int transA, int64_t lda, int64_t i, int64_t k) {
  return transA ? A[k * lda + i] : A[i * lda + k];
}

ORACLE_API void oracle_gemm_f32(int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                                const float* A, int64_t lda, const float* B, int64_t ldb, float beta, float* C,
                                int64_t ldc, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
      for (int64_t j = 0; j < N; ++j) acc[j] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        const float a = a_at_f32(A, transA, lda, i, k);
        if (!transB) {
          const float* brow = B + k * ldb;
          for (int64_t j = 0; j < N; ++j) acc[j] = fmaf(a, brow[j], acc[j]);
        } else {
          for (int64_t j = 0; j < N; ++j) acc[j] = fmaf(a, B[j * ldb + k], acc[j]);
        }
      }
      float* crow = C + i * ldc;
      for (int64_t j = 0; j < N; ++j) crow[j] = axpby_f32(alpha, acc[j], beta, crow[j]);
    }
    free(acc);
  }
}

ORACLE_API void oracle_gemm_f64(int transA, int transB, int64_t M, int64_t N, int64_t K, double alpha,
                                const double* A, int64_t lda, const double* B, int64_t ldb, double beta,
                                double* C, int64_t ldc, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
      for (int64_t j = 0; j < N; ++j) acc[j] = 0.0;
      for (int64_t k = 0; k < K; ++k) {
        const double a = transA ? A[k * lda + i] : A[i * lda + k];
        for (int64_t j = 0; j < N; ++j) acc[j] = fma(a, transB ? B[j * ldb + k] : B[k * ldb + j], acc[j]);
      }
      double* crow = C + i * ldc;
      for (int64_t j = 0; j < N; ++j) crow[j] = beta != 0.0 ? fma(alpha, acc[j], beta * crow[j]) : alpha * acc[j];
    }
    free(acc);
  }
}

/* Fused epilogue of cuopx_gemm_ex, restating MatMulReluFused
 * (src/cuda_op/detail/cuDNN/kernel_fusion.cu:117-136): + bias[col], then
 * ReLU(x) = x if x > 0 else +0.  Flags: 1 = bias, 2 = ReLU.                  */
static inline float epi_f32(float v, const float* bias, int64_t j, int epi) {
  if (epi & 1) v = v + bias[j];
  if (epi & 2) v = v > 0.0f ? v : 0.0f;
  return v;
}

ORACLE_API void oracle_epilogue_f32(int64_t M, int64_t N, float* C, int64_t ldc, const float* bias, int epi) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) C[i * ldc + j] = epi_f32(C[i * ldc + j], bias, j, epi);
}

ORACLE_API void oracle_epilogue_f64(int64_t M, int64_t N, double* C, int64_t ldc, const double* bias, int epi) {
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) {
      double v = C[i * ldc + j];
      if (epi & 1) v = v + bias[j];
      if (epi & 2) v = v > 0.0 ? v : 0.0;
      C[i * ldc + j] = v;
    }
}

/* fp16/bf16 inputs, fp32 fma chain, one RNE rounding (after the optional
 * epilogue; bias is fp16/bf16 bits, widened).  Rows are processed in blocks
 * of RB so each widened B row is reused RB times.                            */
#define RB 8
ORACLE_API void oracle_gemm_lowp_ex(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                                    const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, float beta,
                                    uint16_t* C, int64_t ldc, const uint16_t* bias, int epi, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
  const int64_t nblk = (M + RB - 1) / RB;
#pragma omp parallel num_threads(nthreads)
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)RB * (size_t)(N > 0 ? N : 1));
    float* brow = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(static)
    for (int64_t blk = 0; blk < nblk; ++blk) {
      const int64_t i0 = blk * RB;
      const int64_t rows = (M - i0) < RB ? (M - i0) : RB;
      for (int64_t r = 0; r < rows * N; ++r) acc[r] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        for (int64_t j = 0; j < N; ++j) brow[j] = lowp_to_f32(dtype, transB ? B[j * ldb + k] : B[k * ldb + j]);
        for (int64_t r = 0; r < rows; ++r) {
          const int64_t i = i0 + r;
          const float a = lowp_to_f32(dtype, transA ? A[k * lda + i] : A[i * lda + k]);
          float* ar = acc + r * N;
          for (int64_t j = 0; j < N; ++j) ar[j] = fmaf(a, brow[j], ar[j]);
        }
      }
      for (int64_t r = 0; r < rows; ++r) {
        uint16_t* crow = C + (i0 + r) * ldc;
        const float* ar = acc + r * N;
        for (int64_t j = 0; j < N; ++j) {
          float v = beta != 0.0f ? axpby_f32(alpha, ar[j], beta, lowp_to_f32(dtype, crow[j])) : alpha * ar[j];
          if (epi & 1) v = v + lowp_to_f32(dtype, bias[j]);
          if (epi & 2) v = v > 0.0f ? v : 0.0f;
          crow[j] = f32_to_lowp(dtype, v);
        }
      }
    }
    free(acc);
    free(brow);
  }
}

ORACLE_API void oracle_gemm_lowp(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                                 const uint16_t* A, int64_t lda, const uint16_t* B, int64_t ldb, float beta,
                                 uint16_t* C, int64_t ldc, int nthreads) {
  oracle_gemm_lowp_ex(dtype, transA, transB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, NULL, 0, nthreads);
}

/* Strided batched form of oracle_gemm_lowp / oracle_gemm_f32: batches are
 * spread over the threads (each batch single-threaded), the arithmetic of
 * every batch is the single-GEMM oracle's.                                   */
ORACLE_API void oracle_gemm_batched_lowp(int dtype, int transA, int transB, int64_t M, int64_t N, int64_t K,
                                         float alpha, const uint16_t* A, int64_t lda, int64_t sA,
                                         const uint16_t* B, int64_t ldb, int64_t sB, float beta, uint16_t* C,
                                         int64_t ldc, int64_t sC, int64_t batch, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t b = 0; b < batch; ++b)
    oracle_gemm_lowp(dtype, transA, transB, M, N, K, alpha, A + b * sA, lda, B + b * sB, ldb, beta, C + b * sC, ldc,
                     1);
}

ORACLE_API void oracle_gemm_batched_f32(int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
                                        const float* A, int64_t lda, int64_t sA, const float* B, int64_t ldb,
                                        int64_t sB, float beta, float* C, int64_t ldc, int64_t sC, int64_t batch,
                                        int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t b = 0; b < batch; ++b)
    oracle_gemm_f32(transA, transB, M, N, K, alpha, A + b * sA, lda, B + b * sB, ldb, beta, C + b * sC, ldc, 1);
}

/* fp64-accumulated value of selected outputs (rows[r], cols[c]) of
 * op(A) op(B) for error norms at sizes where a full CPU product is too slow.
 * Inputs are fp32 (already widened); out is [nr][nc].                        */
ORACLE_API void oracle_gemm_sample_f64(int transA, int transB, int64_t K, const float* A, int64_t lda,
                                       const float* B, int64_t ldb, const int64_t* rows, int64_t nr,
                                       const int64_t* cols, int64_t nc, double* out, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < nr; ++r) {
    const int64_t i = rows[r];
    for (int64_t c = 0; c < nc; ++c) {
      const int64_t j = cols[c];
      double s = 0.0;
      for (int64_t k = 0; k < K; ++k)
        s += (double)(transA ? A[k * lda + i] : A[i * lda + k]) * (double)(transB ? B[j * ldb + k] : B[k * ldb + j]);
      out[r * nc + c] = s;
    }
  }
}

/* --------------------------------------------------------------- GEMV --
 * y_i = alpha * sum_j op(A)_ij x_j (+ beta * y_i); trans reads A[j*lda+i].  */
ORACLE_API void oracle_gemv_f32(int trans, int64_t M, int64_t N, float alpha, const float* A, int64_t lda,
                                const float* x, float beta, float* y, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
  if (!trans) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t i = 0; i < M; ++i) {
      const float* arow = A + i * lda;
      float s = 0.0f;
      for (int64_t j = 0; j < N; ++j) s = fmaf(arow[j], x[j], s);
      y[i] = axpby_f32(alpha, s, beta, y[i]);
    }
  } else {
    /* Each thread owns a contiguous range of outputs and walks every row of A
     * over that range; each output's fma chain still runs j = 0..N-1 in order. */
    float* acc = (float*)calloc((size_t)(M > 0 ? M : 1), sizeof(float));
#pragma omp parallel num_threads(nthreads)
    {
#ifdef _OPENMP
      const int64_t nt = omp_get_num_threads(), t = omp_get_thread_num();
#else
      const int64_t nt = 1, t = 0;
#endif
      const int64_t chunk = ((M + nt - 1) / nt + 15) / 16 * 16;
      const int64_t i0 = t * chunk < M ? t * chunk : M;
      const int64_t i1 = i0 + chunk < M ? i0 + chunk : M;
      for (int64_t j = 0; j < N; ++j) {
        const float* arow = A + j * lda;
        const float xj = x[j];
        for (int64_t i = i0; i < i1; ++i) acc[i] = fmaf(arow[i], xj, acc[i]);
      }
      for (int64_t i = i0; i < i1; ++i) y[i] = axpby_f32(alpha, acc[i], beta, y[i]);
    }
    free(acc);
  }
}

ORACLE_API void oracle_gemv_f64acc(int trans, int64_t M, int64_t N, const float* A, int64_t lda, const float* x,
                                   double* out, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    double s = 0.0;
    for (int64_t j = 0; j < N; ++j) s += (double)(trans ? A[j * lda + i] : A[i * lda + j]) * (double)x[j];
    out[i] = s;
  }
}

ORACLE_API int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
