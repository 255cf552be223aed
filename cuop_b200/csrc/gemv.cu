// GEMV kernels: y = alpha * op(A) x + beta * y, row-major A.
//
// Bandwidth-bound design for B200 (no tensor cores):
//  * gemv_n_rows   — one warp per row, 16-byte streaming loads of A spread
//                    across the 32 lanes (fully coalesced), x through L1,
//                    warp-shuffle reduction.  Used when there are enough rows
//                    to fill 148 SMs.
//  * gemv_n_splitk — short-wide shapes: rows split into column chunks over
//                    several CTAs; partial sums go to a workspace and the last
//                    CTA to arrive for a row group reduces them in fixed
//                    chunk order (deterministic, single launch).
//  * gemv_t_splitk — transposed: each thread owns 16 bytes of adjacent
//                    output columns and walks rows (coalesced 16-byte loads),
//                    rows split over CTAs, same last-CTA reduction.
// The streaming kernels in gemv_stream.cu take precedence whenever rows are
// 16-byte aligned (and, for y = A x, x fits eight vectors per lane); these
// kernels cover every other shape.
//
// Math follows the reference kernels: y_i = alpha * sum_j A_ij x_j + beta * y_i
// (src/cuda_op/detail/cuBlas/gemv.cu:10-23; transposed indexing A[col*m+row]
// at gemv.cu:17), accumulated in fp32 (fp64 for double).
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

// 16-byte streaming load of A (read once: do not allocate in L1).
__device__ __forceinline__ uint4 ld_stream_16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, typename AccOf<T>::type (&out)[Vec16<T>::N]) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N; ++i) out[i] = to_acc<T>(e[i]);
}

template <typename T>
__device__ __forceinline__ void store_y(T* y, int64_t i, typename AccOf<T>::type acc, typename AccOf<T>::type alpha,
                                        typename AccOf<T>::type beta) {
  using Acc = typename AccOf<T>::type;
  y[i] = from_acc<T>(beta != Acc(0) ? epi_axpby(alpha, acc, beta, to_acc<T>(y[i])) : epi_scale(alpha, acc));
}

template <typename Acc>
__device__ __forceinline__ Acc warp_sum(Acc v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum of row `row` over columns [c0, c1) by one warp.  When VECTOR, c0, c1,
// the row start and x are 16-byte aligned multiples of the vector width.
template <typename T, bool VECTOR>
__device__ __forceinline__ typename AccOf<T>::type warp_row_dot(const T* __restrict__ arow,
                                                                const T* __restrict__ x, int64_t c0, int64_t c1,
                                                                int lane) {
  using Acc = typename AccOf<T>::type;
  constexpr int V = Vec16<T>::N;
  Acc acc = 0;
  if constexpr (VECTOR) {
    constexpr int U = 4;  // 16-byte loads in flight per lane
    int64_t v = c0 / V + lane;
    const int64_t vend = c1 / V;
    for (; v + 32 * (U - 1) < vend; v += 32 * U) {
      uint4 a[U], b[U];
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = ld_stream_16(arow + (v + 32 * u) * V);
#pragma unroll
      for (int u = 0; u < U; ++u) b[u] = __ldg(reinterpret_cast<const uint4*>(x) + (v + 32 * u));
#pragma unroll
      for (int u = 0; u < U; ++u) {
        Acc fa[V], fb[V];
        unpack16<T>(a[u], fa);
        unpack16<T>(b[u], fb);
#pragma unroll
        for (int i = 0; i < V; ++i) acc = fma(fa[i], fb[i], acc);
      }
    }
    for (; v < vend; v += 32) {
      Acc fa[V], fb[V];
      unpack16<T>(ld_stream_16(arow + v * V), fa);
      unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x) + v), fb);
#pragma unroll
      for (int i = 0; i < V; ++i) acc = fma(fa[i], fb[i], acc);
    }
  } else {
    for (int64_t c = c0 + lane; c < c1; c += 32) acc = fma(to_acc<T>(arow[c]), to_acc<T>(x[c]), acc);
  }
  return warp_sum(acc);
}

// ---------------------------------------------------------------------------
// Non-transposed, one warp per row.
// ---------------------------------------------------------------------------
template <typename T, bool VECTOR>
__global__ void __launch_bounds__(256) gemv_n_rows(int64_t M, int64_t N, typename AccOf<T>::type alpha,
                                                   const T* __restrict__ A, int64_t lda, const T* __restrict__ x,
                                                   typename AccOf<T>::type beta, T* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  auto acc = warp_row_dot<T, VECTOR>(A + row * lda, x, 0, N, lane);
  if (lane == 0) store_y<T>(y, row, acc, alpha, beta);
}

// ---------------------------------------------------------------------------
// Reference-order GEMV (fp32/fp64 in CUOPX_FP32_FFMA mode): one thread per
// output, whose fma chain runs over j = 0..N-1 in ascending order, then the
// reference's epilogue — the arithmetic of the reference's gemv_kernel
// (src/cuda_op/detail/cuBlas/gemv.cu:10-23), so its results are reproduced
// bit for bit.  Exactness, not bandwidth, is the point of this kernel.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) gemv_ordered(int trans, int64_t M, int64_t N, typename AccOf<T>::type alpha,
                                                    const T* __restrict__ A, int64_t lda, const T* __restrict__ x,
                                                    typename AccOf<T>::type beta, T* __restrict__ y) {
  using Acc = typename AccOf<T>::type;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M) return;
  Acc s = 0;
  if (trans) {
    for (int64_t j = 0; j < N; ++j) s = fma(to_acc<T>(A[j * lda + i]), to_acc<T>(x[j]), s);
  } else {
    const T* row = A + i * lda;
    for (int64_t j = 0; j < N; ++j) s = fma(to_acc<T>(row[j]), to_acc<T>(x[j]), s);
  }
  store_y<T>(y, i, s, alpha, beta);
}

// ---------------------------------------------------------------------------
// Split-K last-arrival reduction shared by both split kernels.
// partials: [splits][M] accumulators; counters: one per group.
// Returns true in the (single) CTA that must reduce `group`.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool arrive_and_check_last(unsigned int* counters, int group, unsigned int splits) {
  __shared__ unsigned int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    unsigned int prev = atomicAdd(&counters[group], 1u);
    if (prev >= splits) record_device_error(kDevErrSplitReduce);
    s_last = (prev == splits - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last != 0;
}

// Non-transposed split-K: blockDim = 256 (8 warps = 8 rows), grid = (row groups, splits).
template <typename T, bool VECTOR>
__global__ void __launch_bounds__(256) gemv_n_splitk(int64_t M, int64_t N, typename AccOf<T>::type alpha,
                                                     const T* __restrict__ A, int64_t lda,
                                                     const T* __restrict__ x, typename AccOf<T>::type beta,
                                                     T* __restrict__ y, int64_t chunk,
                                                     typename AccOf<T>::type* __restrict__ partials,
                                                     unsigned int* __restrict__ counters) {
  using Acc = typename AccOf<T>::type;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int group = blockIdx.x;
  const unsigned int splits = gridDim.y;
  const int64_t row = static_cast<int64_t>(group) * 8 + warp;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * chunk;
  const int64_t c1 = min(N, c0 + chunk);
  if (row < M) {
    Acc acc = warp_row_dot<T, VECTOR>(A + row * lda, x, c0, c1, lane);
    if (lane == 0) partials[static_cast<int64_t>(blockIdx.y) * M + row] = acc;
  }
  if (!arrive_and_check_last(counters, group, splits)) return;
  if (row < M && lane == 0) {
    Acc acc = 0;
    for (unsigned int s = 0; s < splits; ++s) acc += __ldcg(&partials[static_cast<int64_t>(s) * M + row]);
    store_y<T>(y, row, acc, alpha, beta);
  }
  if (threadIdx.x == 0) counters[group] = 0u;
}

// Transposed split-K: blockDim = (TX, TY); each thread owns V adjacent output
// columns; grid = (column strips, row chunks).
template <typename T, bool VECTOR>
__global__ void __launch_bounds__(256) gemv_t_splitk(int64_t M, int64_t N, typename AccOf<T>::type alpha,
                                                     const T* __restrict__ A, int64_t lda,
                                                     const T* __restrict__ x, typename AccOf<T>::type beta,
                                                     T* __restrict__ y, int64_t chunk,
                                                     typename AccOf<T>::type* __restrict__ partials,
                                                     unsigned int* __restrict__ counters) {
  using Acc = typename AccOf<T>::type;
  constexpr int V = Vec16<T>::N;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Acc* red = reinterpret_cast<Acc*>(smem_raw);  // [TY][TX][V]

  const int tx = threadIdx.x, ty = threadIdx.y;
  const int TX = blockDim.x, TY = blockDim.y;
  const unsigned int splits = gridDim.y;
  const int64_t col0 = (static_cast<int64_t>(blockIdx.x) * TX + tx) * V;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * chunk;
  const int64_t r1 = min(N, r0 + chunk);

  Acc acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0;

  if (col0 < M) {
    if constexpr (VECTOR) {
      constexpr int U = 4;
      int64_t r = r0 + ty;
      for (; r + static_cast<int64_t>(TY) * (U - 1) < r1; r += static_cast<int64_t>(TY) * U) {
        uint4 a[U];
        Acc xv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) a[u] = ld_stream_16(A + (r + static_cast<int64_t>(TY) * u) * lda + col0);
#pragma unroll
        for (int u = 0; u < U; ++u) xv[u] = to_acc<T>(x[r + static_cast<int64_t>(TY) * u]);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          Acc fa[V];
          unpack16<T>(a[u], fa);
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] = fma(fa[i], xv[u], acc[i]);
        }
      }
      for (; r < r1; r += TY) {
        Acc fa[V];
        unpack16<T>(ld_stream_16(A + r * lda + col0), fa);
        const Acc xr = to_acc<T>(x[r]);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = fma(fa[i], xr, acc[i]);
      }
    } else {
      for (int64_t r = r0 + ty; r < r1; r += TY) {
        const Acc xr = to_acc<T>(x[r]);
#pragma unroll
        for (int i = 0; i < V; ++i)
          if (col0 + i < M) acc[i] = fma(to_acc<T>(A[r * lda + col0 + i]), xr, acc[i]);
      }
    }
  }

  // Reduce over ty in fixed order.
  if (TY > 1) {
#pragma unroll
    for (int i = 0; i < V; ++i) red[(ty * TX + tx) * V + i] = acc[i];
    __syncthreads();
    if (ty == 0) {
      for (int j = 1; j < TY; ++j)
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] += red[(j * TX + tx) * V + i];
    }
  }

  if (splits == 1) {
    if (ty == 0)
#pragma unroll
      for (int i = 0; i < V; ++i)
        if (col0 + i < M) store_y<T>(y, col0 + i, acc[i], alpha, beta);
    return;
  }

  if (ty == 0)
#pragma unroll
    for (int i = 0; i < V; ++i)
      if (col0 + i < M) partials[static_cast<int64_t>(blockIdx.y) * M + col0 + i] = acc[i];
  if (!arrive_and_check_last(counters, blockIdx.x, splits)) return;
  if (ty == 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      if (col0 + i < M) {
        Acc s = 0;
        for (unsigned int k = 0; k < splits; ++k) s += __ldcg(&partials[static_cast<int64_t>(k) * M + col0 + i]);
        store_y<T>(y, col0 + i, s, alpha, beta);
      }
    }
  }
  if (tx == 0 && ty == 0) counters[blockIdx.x] = 0u;
}

// ---------------------------------------------------------------------------
// Host-side planning + launch.
// ---------------------------------------------------------------------------
namespace {

struct GemvPlan {
  int variant;  // 0 rows, 1 n-splitk, 2 t-splitk
  bool vector;
  int64_t groups;  // grid.x
  int64_t splits;  // grid.y
  int64_t chunk;
  int tx, ty;
  size_t partial_bytes;
  size_t counter_bytes;
};

constexpr size_t kAlign = 256;
// Workspace layout (fixed, so any earlier call's partials can never land on
// a later call's counters): [kMaxCounters arrival counters][partial sums].
constexpr int64_t kMaxCounters = 4096;
constexpr size_t kCounterBytes = kMaxCounters * sizeof(unsigned int);
inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <typename T>
GemvPlan plan_gemv(int trans, int64_t M, int64_t N, int64_t lda, const void* A, const void* x, int num_sms) {
  using Acc = typename AccOf<T>::type;
  constexpr int V = Vec16<T>::N;
  GemvPlan p{};
  const int64_t target_ctas = static_cast<int64_t>(num_sms) * 4;
  const bool a_al = (reinterpret_cast<uintptr_t>(A) % 16 == 0) && ((lda * (int64_t)sizeof(T)) % 16 == 0);
  if (!trans) {
    p.vector = a_al && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (N % V == 0);
    const int64_t groups = (M + 7) / 8;
    if (groups >= target_ctas / 2 || N < 32 * V * 8) {
      p.variant = 0;
      p.groups = groups;
      p.splits = 1;
    } else {
      p.variant = 1;
      p.groups = groups;
      int64_t splits = (target_ctas + groups - 1) / groups;
      const int64_t min_chunk = 32 * V * 4;  // one unrolled sweep of the warp
      splits = std::max<int64_t>(1, std::min<int64_t>(splits, N / min_chunk));
      int64_t chunk = (N + splits - 1) / splits;
      chunk = (chunk + V - 1) / V * V;  // keep chunk starts vector-aligned
      p.splits = (N + chunk - 1) / chunk;
      p.chunk = chunk;
      if (p.splits <= 1) {
        p.variant = 0;
        p.splits = 1;
      }
    }
  } else {
    p.variant = 2;
    p.vector = a_al && (M % V == 0);
    const int64_t colvecs = (M + V - 1) / V;
    int tx = 256;
    while (tx > 8 && tx / 2 >= colvecs) tx /= 2;
    p.tx = tx;
    p.ty = 256 / tx;
    p.groups = (colvecs + tx - 1) / tx;
    int64_t splits = (target_ctas + p.groups - 1) / p.groups;
    const int64_t min_rows = static_cast<int64_t>(p.ty) * 16;
    splits = std::max<int64_t>(1, std::min<int64_t>(splits, (N + min_rows - 1) / min_rows));
    p.chunk = std::max<int64_t>(1, (N + splits - 1) / splits);
    p.splits = std::max<int64_t>(1, (N + p.chunk - 1) / p.chunk);
  }
  if (p.splits > 1 && p.groups > kMaxCounters) {  // enough CTAs without splitting
    if (!trans) {
      p.variant = 0;
      p.groups = (M + 7) / 8;
    }
    p.splits = 1;
    p.chunk = std::max<int64_t>(N, 1);
  }
  if (p.splits > 1) {
    p.counter_bytes = kCounterBytes;
    p.partial_bytes = round_up(static_cast<size_t>(p.splits) * M * sizeof(Acc), kAlign);
  }
  return p;
}

template <typename T>
int launch_gemv(int trans, int64_t M, int64_t N, double alpha_d, const void* A_, int64_t lda, const void* x_,
                double beta_d, void* y_, void* ws, size_t ws_bytes, cudaStream_t stream) {
  using Acc = typename AccOf<T>::type;
  const T* A = static_cast<const T*>(A_);
  const T* x = static_cast<const T*>(x_);
  T* y = static_cast<T*>(y_);
  const Acc alpha = static_cast<Acc>(alpha_d), beta = static_cast<Acc>(beta_d);
  if constexpr (sizeof(Acc) == sizeof(T)) {  // fp32 / fp64 in FFMA mode: the reference's order
    if (fp32_mode() == CUOPX_FP32_FFMA) {
      gemv_ordered<T><<<static_cast<unsigned>((M + 255) / 256), 256, 0, stream>>>(trans, M, N, alpha, A, lda, x,
                                                                                    beta, y);
      note_launch("gemv_ordered");
      return check_launch();
    }
  }
  // Streaming kernels (gemv_stream.cu) first; the kernels below cover the
  // shapes and alignments they do not take.
  const int rs = launch_gemv_stream<T>(trans, M, N, alpha_d, A_, lda, x_, beta_d, y_, ws, ws_bytes, kCounterBytes,
                                       stream);
  if (rs >= 0) return rs;
  GemvPlan p = plan_gemv<T>(trans, M, N, lda, A_, x_, device_sm_count());
  const size_t need = p.partial_bytes + p.counter_bytes;
  if (p.splits > 1 && (ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) % kAlign) != 0)) {
    // Not enough scratch: single-pass variants (correct, fewer CTAs in flight).
    if (!trans) {
      p.variant = 0;
      p.splits = 1;
      p.groups = (M + 7) / 8;
    } else {
      p.splits = 1;
      p.chunk = std::max<int64_t>(N, 1);
    }
  }
  unsigned int* counters = reinterpret_cast<unsigned int*>(ws);
  Acc* partials = reinterpret_cast<Acc*>(static_cast<char*>(ws) + kCounterBytes);
  if (p.variant == 0) {
    dim3 grid(static_cast<unsigned>((M + 7) / 8));
    if (p.vector)
      gemv_n_rows<T, true><<<grid, 256, 0, stream>>>(M, N, alpha, A, lda, x, beta, y);
    else
      gemv_n_rows<T, false><<<grid, 256, 0, stream>>>(M, N, alpha, A, lda, x, beta, y);
    note_launch("gemv_n_rows");
  } else if (p.variant == 1) {
    dim3 grid(static_cast<unsigned>(p.groups), static_cast<unsigned>(p.splits));
    if (p.vector)
      gemv_n_splitk<T, true><<<grid, 256, 0, stream>>>(M, N, alpha, A, lda, x, beta, y, p.chunk, partials, counters);
    else
      gemv_n_splitk<T, false><<<grid, 256, 0, stream>>>(M, N, alpha, A, lda, x, beta, y, p.chunk, partials,
                                                        counters);
    note_launch("gemv_n_splitk");
  } else {
    dim3 grid(static_cast<unsigned>(p.groups), static_cast<unsigned>(p.splits));
    dim3 block(p.tx, p.ty);
    const size_t smem = (p.ty > 1) ? static_cast<size_t>(p.tx) * p.ty * Vec16<T>::N * sizeof(Acc) : 0;
    if (p.vector)
      gemv_t_splitk<T, true><<<grid, block, smem, stream>>>(M, N, alpha, A, lda, x, beta, y, p.chunk, partials,
                                                            counters);
    else
      gemv_t_splitk<T, false><<<grid, block, smem, stream>>>(M, N, alpha, A, lda, x, beta, y, p.chunk, partials,
                                                             counters);
    note_launch(p.splits > 1 ? "gemv_t_splitk" : "gemv_t_single");
  }
  return check_launch();
}

}  // namespace

size_t gemv_workspace_size(int dtype, int trans, int64_t M, int64_t N) {
  GemvPlan p{};
  // Alignment is assumed favourable for sizing; the split count does not depend on it.
  const void* al = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  const int sms = device_sm_count();
  switch (dtype) {
    case CUOPX_F32: p = plan_gemv<float>(trans, M, N, trans ? M : N, al, al, sms); break;
    case CUOPX_F64: p = plan_gemv<double>(trans, M, N, trans ? M : N, al, al, sms); break;
    case CUOPX_F16: p = plan_gemv<__half>(trans, M, N, trans ? M : N, al, al, sms); break;
    case CUOPX_BF16: p = plan_gemv<__nv_bfloat16>(trans, M, N, trans ? M : N, al, al, sms); break;
    default: return 0;
  }
  const size_t stream_ws = gemv_stream_workspace(dtype, trans, M, N);
  return std::max(p.partial_bytes + p.counter_bytes, stream_ws ? stream_ws + kCounterBytes : size_t(0));
}

int gemv_dispatch(int dtype, int trans, int64_t M, int64_t N, double alpha, const void* A, int64_t lda,
                  const void* x, double beta, void* y, void* ws, size_t ws_bytes, cudaStream_t stream) {
  switch (dtype) {
    case CUOPX_F32: return launch_gemv<float>(trans, M, N, alpha, A, lda, x, beta, y, ws, ws_bytes, stream);
    case CUOPX_F64: return launch_gemv<double>(trans, M, N, alpha, A, lda, x, beta, y, ws, ws_bytes, stream);
    case CUOPX_F16: return launch_gemv<__half>(trans, M, N, alpha, A, lda, x, beta, y, ws, ws_bytes, stream);
    case CUOPX_BF16:
      return launch_gemv<__nv_bfloat16>(trans, M, N, alpha, A, lda, x, beta, y, ws, ws_bytes, stream);
    default: return CUOPX_UNSUPPORTED_TYPE;
  }
}

}  // namespace cuopx
