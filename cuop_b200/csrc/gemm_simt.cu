// SIMT GEMM back-ends.
//
// * gemm_generic_kernel — any dtype (f32/f64/f16/bf16), any transpose and
//   leading dimension, strided batch, ragged edges.  64x64 CTA tile, 4x4
//   outputs per thread.  Covers shapes the TMA/tcgen05 path cannot take
//   (unaligned strides, tiny problems, fp64).
// * gemm_f32_kernel<BM,BN> — register-blocked fp32 FFMA kernel for the
//   non-transposed layout with 16-byte aligned rows: BMxBNx8 tiles,
//   double-buffered shared memory with register prefetch, up to 8x8
//   outputs per thread.
//
// Both accumulate every output as one fused-multiply-add chain over k in
// ascending order, then apply C = fma(alpha, acc, beta*C) (alpha*acc when
// beta == 0; then the optional bias add and ReLU of cuopx_gemm_ex) — the
// reference kernels' summation order and epilogue (src/cuda_op/detail/cuBlas/
// gemm.cu:23-41, gemm.cu:264-291) — so fp32 results reproduce the reference's
// own kernels, and a CPU loop doing the same fmaf chain, bit for bit.
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

template <typename T>
__device__ __forceinline__ typename AccOf<T>::type epilogue_value(typename AccOf<T>::type acc,
                                                                  typename AccOf<T>::type alpha,
                                                                  typename AccOf<T>::type beta, const T* c) {
  using Acc = typename AccOf<T>::type;
  return beta != Acc(0) ? epi_axpby(alpha, acc, beta, to_acc<T>(*c)) : epi_scale(alpha, acc);
}

// ---------------------------------------------------------------------------
// Generic kernel.
// ---------------------------------------------------------------------------
constexpr int GT = 64;  // tile
constexpr int GK = 16;  // k tile

template <typename T>
__global__ void __launch_bounds__(256) gemm_generic_kernel(GemmProblem p) {
  using Acc = typename AccOf<T>::type;
  __shared__ Acc As[GK][GT + 1];
  __shared__ Acc Bs[GK][GT + 1];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * GT;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * GT;
  const Acc alpha = static_cast<Acc>(p.alpha), beta = static_cast<Acc>(p.beta);

  for (int64_t b = blockIdx.z; b < p.batch; b += gridDim.z) {
    const T* A = static_cast<const T*>(p.A) + b * p.strideA;
    const T* B = static_cast<const T*>(p.B) + b * p.strideB;
    T* C = static_cast<T*>(p.C) + b * p.strideC;
    Acc acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0;

    for (int64_t k0 = 0; k0 < p.K; k0 += GK) {
      // A tile: GT rows (m) x GK (k); B tile: GK (k) x GT cols (n).
      for (int idx = tid; idx < GT * GK; idx += 256) {
        int mi, ki;
        if (p.transA) {  // A stored K x M: walk m fastest for coalescing
          mi = idx % GT;
          ki = idx / GT;
        } else {
          ki = idx % GK;
          mi = idx / GK;
        }
        const int64_t gm = m0 + mi, gk = k0 + ki;
        Acc v = 0;
        if (gm < p.M && gk < p.K) v = to_acc<T>(p.transA ? A[gk * p.lda + gm] : A[gm * p.lda + gk]);
        As[ki][mi] = v;
      }
      for (int idx = tid; idx < GT * GK; idx += 256) {
        int ni, ki;
        if (p.transB) {  // B stored N x K
          ki = idx % GK;
          ni = idx / GK;
        } else {
          ni = idx % GT;
          ki = idx / GT;
        }
        const int64_t gn = n0 + ni, gk = k0 + ki;
        Acc v = 0;
        if (gn < p.N && gk < p.K) v = to_acc<T>(p.transB ? B[gn * p.ldb + gk] : B[gk * p.ldb + gn]);
        Bs[ki][ni] = v;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < GK; ++kk) {
        Acc a[4], bb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], bb[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty + 16 * i;
      if (gm >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx + 16 * j;
        if (gn >= p.N) continue;
        T* c = C + gm * p.ldc + gn;
        *c = from_acc<T>(apply_epilogue<T>(epilogue_value<T>(acc[i][j], alpha, beta, c), p.bias, gn, p.epi));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Register-blocked fp32 kernel (non-transposed, 16-byte aligned rows).
// ---------------------------------------------------------------------------
template <int BM, int BN>
__global__ void __launch_bounds__(256) gemm_f32_kernel(GemmProblem p) {
  constexpr int BK = 8;
  constexpr int TM = BM / 16, TN = BN / 16;  // outputs per thread
  constexpr int HM = TM / 4, HN = TN / 4;    // 4-wide sub-blocks, 64 apart
  constexpr int A_LD = BM * 2 / 256 > 0 ? BM * 2 / 256 : 1;  // float4 loads per thread (may be idle)
  constexpr int B_LD = BN * 2 / 256 > 0 ? BN * 2 / 256 : 1;
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
  const float alpha = static_cast<float>(p.alpha), beta = static_cast<float>(p.beta);

  for (int64_t b = blockIdx.z; b < p.batch; b += gridDim.z) {
    const float* A = static_cast<const float*>(p.A) + b * p.strideA;
    const float* B = static_cast<const float*>(p.B) + b * p.strideB;
    float* C = static_cast<float*>(p.C) + b * p.strideC;

    float4 ra[A_LD], rb[B_LD];
    auto load_tiles = [&](int64_t k0) {
#pragma unroll
      for (int l = 0; l < A_LD; ++l) {
        const int idx = tid + l * 256;
        const int row = idx / 2, kq = (idx % 2) * 4;
        const int64_t gm = m0 + row, gk = k0 + kq;
        ra[l] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (idx < BM * 2 && gm < p.M && gk < p.K) ra[l] = *reinterpret_cast<const float4*>(A + gm * p.lda + gk);
      }
#pragma unroll
      for (int l = 0; l < B_LD; ++l) {
        const int idx = tid + l * 256;
        const int krow = idx / (BN / 4), nq = (idx % (BN / 4)) * 4;
        const int64_t gk = k0 + krow, gn = n0 + nq;
        rb[l] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (idx < BN * 2 && gk < p.K && gn < p.N) rb[l] = *reinterpret_cast<const float4*>(B + gk * p.ldb + gn);
      }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
      for (int l = 0; l < A_LD; ++l) {
        const int idx = tid + l * 256;
        if (idx < BM * 2) {
          const int row = idx / 2, kq = (idx % 2) * 4;
          As[buf][kq + 0][row] = ra[l].x;
          As[buf][kq + 1][row] = ra[l].y;
          As[buf][kq + 2][row] = ra[l].z;
          As[buf][kq + 3][row] = ra[l].w;
        }
      }
#pragma unroll
      for (int l = 0; l < B_LD; ++l) {
        const int idx = tid + l * 256;
        if (idx < BN * 2) {
          const int krow = idx / (BN / 4), nq = (idx % (BN / 4)) * 4;
          *reinterpret_cast<float4*>(&Bs[buf][krow][nq]) = rb[l];
        }
      }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    const int64_t nk = (p.K + BK - 1) / BK;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    for (int64_t kt = 0; kt < nk; ++kt) {
      const int buf = static_cast<int>(kt & 1);
      if (kt + 1 < nk) load_tiles((kt + 1) * BK);
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float a[TM], bb[TN];
#pragma unroll
        for (int h = 0; h < HM; ++h) {
          const float4 v = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + 64 * h]);
          a[h * 4 + 0] = v.x;
          a[h * 4 + 1] = v.y;
          a[h * 4 + 2] = v.z;
          a[h * 4 + 3] = v.w;
        }
#pragma unroll
        for (int g = 0; g < HN; ++g) {
          const float4 v = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + 64 * g]);
          bb[g * 4 + 0] = v.x;
          bb[g * 4 + 1] = v.y;
          bb[g * 4 + 2] = v.z;
          bb[g * 4 + 3] = v.w;
        }
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
      }
      if (kt + 1 < nk) store_tiles(buf ^ 1);
      __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t gm = m0 + ty * 4 + (i % 4) + 64 * (i / 4);
      if (gm >= p.M) continue;
#pragma unroll
      for (int g = 0; g < HN; ++g) {
        const int64_t gn = n0 + tx * 4 + 64 * g;
        if (gn >= p.N) continue;  // N % 4 == 0 on this path: all 4 or none
        float* c = C + gm * p.ldc + gn;
        float4 out;
        float* o = &out.x;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = apply_epilogue<float>(epilogue_value<float>(acc[i][g * 4 + j], alpha, beta, c + j), p.bias, gn + j,
                                       p.epi);
        *reinterpret_cast<float4*>(c) = out;
      }
    }
  }
}

}  // namespace

int gemm_simt_generic(const GemmProblem& p, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((p.N + GT - 1) / GT), static_cast<unsigned>((p.M + GT - 1) / GT),
            static_cast<unsigned>(std::min<int64_t>(p.batch, 65535)));
  switch (p.dtype) {
    case CUOPX_F32: gemm_generic_kernel<float><<<grid, 256, 0, stream>>>(p); break;
    case CUOPX_F64: gemm_generic_kernel<double><<<grid, 256, 0, stream>>>(p); break;
    case CUOPX_F16: gemm_generic_kernel<__half><<<grid, 256, 0, stream>>>(p); break;
    case CUOPX_BF16: gemm_generic_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p); break;
    default: return CUOPX_UNSUPPORTED_TYPE;
  }
  note_launch("gemm_simt_generic");
  return check_launch();
}

bool gemm_simt_f32_supported(const GemmProblem& p) {
  if (p.dtype != CUOPX_F32 || p.transA || p.transB) return false;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
  return al16(p.A) && al16(p.B) && al16(p.C) && p.K % 4 == 0 && p.N % 4 == 0 && p.lda % 4 == 0 &&
         p.ldb % 4 == 0 && p.ldc % 4 == 0 && (p.batch == 1 || (p.strideA % 4 == 0 && p.strideB % 4 == 0 &&
                                                                  p.strideC % 4 == 0));
}

int gemm_simt_f32(const GemmProblem& p, cudaStream_t stream) {
  // Pick the largest tile that still gives >= one CTA per SM.
  const int sms = device_sm_count();
  auto ctas = [&](int bm, int bn) { return ((p.M + bm - 1) / bm) * ((p.N + bn - 1) / bn) * p.batch; };
  const unsigned gz = static_cast<unsigned>(std::min<int64_t>(p.batch, 65535));
  if (ctas(128, 128) >= sms) {
    dim3 grid(static_cast<unsigned>((p.N + 127) / 128), static_cast<unsigned>((p.M + 127) / 128), gz);
    gemm_f32_kernel<128, 128><<<grid, 256, 0, stream>>>(p);
    note_launch("gemm_f32_128x128");
  } else if (ctas(128, 64) >= sms) {
    dim3 grid(static_cast<unsigned>((p.N + 63) / 64), static_cast<unsigned>((p.M + 127) / 128), gz);
    gemm_f32_kernel<128, 64><<<grid, 256, 0, stream>>>(p);
    note_launch("gemm_f32_128x64");
  } else {
    dim3 grid(static_cast<unsigned>((p.N + 63) / 64), static_cast<unsigned>((p.M + 63) / 64), gz);
    gemm_f32_kernel<64, 64><<<grid, 256, 0, stream>>>(p);
    note_launch("gemm_f32_64x64");
  }
  return check_launch();
}

}  // namespace cuopx
