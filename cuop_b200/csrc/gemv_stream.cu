// Streaming GEMV kernels sized for B200 HBM3e.
//
// Measured on this part (1 GiB read probe): plain 16-byte loads from two
// 256..1024-thread CTAs per SM with 4-16 loads in flight per thread sustain
// ~6.3 TB/s, while TMA bulk copies of 8 KB stall near 4.8 TB/s and 32 KB
// bulk copies whose slots are then read back from shared memory reach ~6.0.
// Both kernels below therefore stream A with ld.global.nc (L1 no-allocate)
// and keep 16 loads of 16 bytes in flight per thread, two 256-thread CTAs
// per SM.
//
// gemv_n_xreg (y = A x): CTA c owns rows [c*R, (c+1)*R); warp w owns the fixed
//   column slice [w*32*KV, (w+1)*32*KV) vectors, so its slice of x lives in
//   registers for the whole kernel.  Each warp reduces its slice of two rows
//   at a time (fma chains per lane, then a butterfly shuffle); the 8 warp
//   partials of each row are added in warp order from shared memory.
// gemv_t_lsu (y = A^T x, A is N x M): the grid is (column strips) x (row
//   splits); a strip is 64 16-byte column groups wide and each group is
//   walked by 4 threads (row phases), 16 rows in flight each.  Split partials
//   go to the workspace and the last CTA of a strip adds them, so narrow
//   strips keep that final, serial step short.
// Both are deterministic: summation order depends only on the shape.
//
// Math: y_i = alpha * sum_j op(A)_ij x_j + beta * y_i (the reference's gemv
// kernels, src/cuda_op/detail/cuBlas/gemv.cu:10-23; transposed indexing
// A[col*m+row], gemv.cu:17), fp32 accumulation (fp64 for double).
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int GS_THREADS = 256;
constexpr int GS_WARPS = GS_THREADS / 32;
constexpr int GS_ROWS_MAX = 64;  // rows per CTA in gemv_n_xreg
constexpr int GS_T_UNROLL = 16;  // rows in flight per thread in gemv_t_lsu
constexpr int GS_T_SV = 64;      // 16-byte column groups per gemv_t_lsu strip
constexpr int GS_T_PHASES = GS_THREADS / GS_T_SV;  // row phases per strip
constexpr int GS_T_WAVES = 1;    // gemv_t_lsu CTAs per resident slot
// Final split reduction: partial vectors loaded together per round, sized so
// they take 64 registers (16 for fp32 / fp64, 8 for 16-bit types).
constexpr int GS_T_RED_REGS = 64;

// Rows of A each CTA asks L2 to fetch before waiting for the previous kernel
// on the stream (programmatic dependent launch): the launch then starts on
// L2 hits while the previous grid's last CTAs still drain.  A prefetch only
// warms L2, the device's point of coherence, so it cannot return data from
// before the previous kernel's writes.
constexpr int GS_N_PREFETCH_ROWS = 2;  // gemv_n_xreg: first rows of the CTA's block
constexpr bool GS_T_PREFETCH = true;   // gemv_t_lsu: first batch of each thread's rows

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ uint4 ld_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename T>
__device__ __forceinline__ void unpack_v(const uint4& v, typename AccOf<T>::type* out) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 16 / (int)sizeof(T); ++i) out[i] = to_acc<T>(e[i]);
}

template <typename Acc>
__device__ __forceinline__ Acc warp_allsum(Acc v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
template <typename T, int KV>
__global__ void __launch_bounds__(GS_THREADS, 2)
    gemv_n_xreg(int64_t M, int64_t N, typename AccOf<T>::type alpha, const T* __restrict__ A, int64_t lda,
                const T* __restrict__ x, typename AccOf<T>::type beta, T* __restrict__ y, int rows_per_cta) {
  using Acc = typename AccOf<T>::type;
  constexpr int V = 16 / sizeof(T);
  __shared__ Acc part[GS_ROWS_MAX][GS_WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nvec = N / V;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int64_t r1 = min(M, r0 + rows_per_cta);
  if ((lane & 7) == 0) {  // one request per 128-byte line of the warp's slice
    for (int64_t r = r0; r < min(r1, r0 + GS_N_PREFETCH_ROWS); ++r) {
      const uint4* a = reinterpret_cast<const uint4*>(A + r * lda) + static_cast<int64_t>(warp) * 32 * KV + lane;
#pragma unroll
      for (int k = 0; k < KV; ++k)
        if (static_cast<int64_t>(warp) * 32 * KV + k * 32 + lane < nvec) prefetch_l2(a + k * 32);
    }
  }
  // The next kernel may start launching once every CTA of this grid has
  // started (its CTAs then take slots freed by exiting CTAs and wait for
  // this grid's completion before touching memory).
  grid_dependency_wait();
  grid_launch_dependents();
  if (r0 >= r1) return;

  Acc xr[KV][V];
  bool valid[KV];
#pragma unroll
  for (int k = 0; k < KV; ++k) {
    const int64_t vi = static_cast<int64_t>(warp) * 32 * KV + k * 32 + lane;
    valid[k] = vi < nvec;
    if (valid[k]) {
      unpack_v<T>(__ldg(reinterpret_cast<const uint4*>(x) + vi), xr[k]);
    } else {
#pragma unroll
      for (int i = 0; i < V; ++i) xr[k][i] = 0;
    }
  }
  const int64_t vbase = static_cast<int64_t>(warp) * 32 * KV + lane;

  int64_t r = r0;
  for (; r + 1 < r1; r += 2) {
    const uint4* a0 = reinterpret_cast<const uint4*>(A + r * lda) + vbase;
    const uint4* a1 = reinterpret_cast<const uint4*>(A + (r + 1) * lda) + vbase;
    uint4 v0[KV], v1[KV];
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      v0[k] = valid[k] ? ld_nc16(a0 + k * 32) : make_uint4(0, 0, 0, 0);
      v1[k] = valid[k] ? ld_nc16(a1 + k * 32) : make_uint4(0, 0, 0, 0);
    }
    Acc s0 = 0, s1 = 0;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      Acc f0[V], f1[V];
      unpack_v<T>(v0[k], f0);
      unpack_v<T>(v1[k], f1);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        s0 = fma(f0[i], xr[k][i], s0);
        s1 = fma(f1[i], xr[k][i], s1);
      }
    }
    s0 = warp_allsum(s0);
    s1 = warp_allsum(s1);
    if (lane == 0) {
      part[r - r0][warp] = s0;
      part[r + 1 - r0][warp] = s1;
    }
  }
  if (r < r1) {
    const uint4* a0 = reinterpret_cast<const uint4*>(A + r * lda) + vbase;
    uint4 v0[KV];
#pragma unroll
    for (int k = 0; k < KV; ++k) v0[k] = valid[k] ? ld_nc16(a0 + k * 32) : make_uint4(0, 0, 0, 0);
    Acc s0 = 0;
#pragma unroll
    for (int k = 0; k < KV; ++k) {
      Acc f0[V];
      unpack_v<T>(v0[k], f0);
#pragma unroll
      for (int i = 0; i < V; ++i) s0 = fma(f0[i], xr[k][i], s0);
    }
    s0 = warp_allsum(s0);
    if (lane == 0) part[r - r0][warp] = s0;
  }
  __syncthreads();
  for (int64_t rr = threadIdx.x; rr < r1 - r0; rr += GS_THREADS) {
    Acc s = part[rr][0];
#pragma unroll
    for (int w = 1; w < GS_WARPS; ++w) s += part[rr][w];
    y[r0 + rr] = from_acc<T>(beta != Acc(0) ? epi_axpby(alpha, s, beta, to_acc<T>(y[r0 + rr])) : epi_scale(alpha, s));
  }
}

// ---------------------------------------------------------------------------
// Thread t of a gemv_t_lsu CTA owns column group t % GS_T_SV of its strip and
// row phase t / GS_T_SV: it walks rows j0 + phase, j0 + phase + GS_T_PHASES,
// ... of the split.  The phases are added in order through shared memory, so
// a strip is only GS_T_SV 16-byte groups wide and the last CTA of a strip has
// splits x GS_T_SV x 16 bytes of partials to add, not a whole-CTA-wide slab.
template <typename T>
__global__ void __launch_bounds__(GS_THREADS, 2)
    gemv_t_lsu(int64_t M, int64_t N, typename AccOf<T>::type alpha, const T* __restrict__ A, int64_t lda,
               const T* __restrict__ x, typename AccOf<T>::type beta, T* __restrict__ y, int64_t rows_per_split,
               typename AccOf<T>::type* __restrict__ partials, unsigned int* __restrict__ counters) {
  using Acc = typename AccOf<T>::type;
  constexpr int V = 16 / sizeof(T);
  constexpr int U = GS_T_UNROLL;
  constexpr int P = GS_T_PHASES;
  constexpr int64_t STRIP = static_cast<int64_t>(GS_T_SV) * V;  // columns per strip
  __shared__ Acc s_phase[P - 1][GS_T_SV * V];
  __shared__ unsigned int s_last;
  const int tid = threadIdx.x;
  const int cv = tid % GS_T_SV, ph = tid / GS_T_SV;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * STRIP + static_cast<int64_t>(cv) * V;
  const bool has = col < M;  // M % V == 0: the group is all in or all out
  const int64_t j0 = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  const int64_t j1 = min(N, j0 + rows_per_split);
  const unsigned int splits = gridDim.y;
  if (GS_T_PREFETCH && has && (tid & 7) == 0) {  // one request per 128-byte line
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (j0 + ph + u * P < j1) prefetch_l2(A + col + (j0 + ph + u * P) * lda);
  }
  grid_dependency_wait();
  grid_launch_dependents();

  Acc acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0;

  if (has) {
    const T* ap = A + col;
    int64_t j = j0 + ph;
    for (; j + (U - 1) * P < j1; j += U * P) {
      uint4 v[U];
      Acc xv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = ld_nc16(ap + (j + u * P) * lda);
#pragma unroll
      for (int u = 0; u < U; ++u) xv[u] = to_acc<T>(__ldg(x + j + u * P));
#pragma unroll
      for (int u = 0; u < U; ++u) {
        Acc f[V];
        unpack_v<T>(v[u], f);
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = fma(f[i], xv[u], acc[i]);
      }
    }
    if (j < j1) {
      // Remainder (< U rows of this phase): one predicated batch, all loads
      // in flight at once, added in the same ascending row order.
      uint4 v[U];
      Acc xv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool in = j + u * P < j1;
        v[u] = in ? ld_nc16(ap + (j + u * P) * lda) : make_uint4(0, 0, 0, 0);
        xv[u] = in ? to_acc<T>(__ldg(x + j + u * P)) : Acc(0);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (j + u * P < j1) {
          Acc f[V];
          unpack_v<T>(v[u], f);
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] = fma(f[i], xv[u], acc[i]);
        }
      }
    }
  }
  // Phase 0 adds phases 1..P-1 in order.
  if (ph > 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) s_phase[ph - 1][cv * V + i] = acc[i];
  }
  __syncthreads();
  if (ph == 0) {
#pragma unroll
    for (int q = 0; q < P - 1; ++q)
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += s_phase[q][cv * V + i];
  }

  if (splits == 1) {
    if (ph == 0 && has) {
#pragma unroll
      for (int i = 0; i < V; ++i) {
        y[col + i] =
            from_acc<T>(beta != Acc(0) ? epi_axpby(alpha, acc[i], beta, to_acc<T>(y[col + i])) : epi_scale(alpha, acc[i]));
      }
    }
    return;
  }
  // V partials of one split are V * sizeof(Acc) contiguous, 16-byte aligned
  // bytes (M % V == 0, 256-byte aligned workspace): vector stores and loads.
  constexpr int QN = V * static_cast<int>(sizeof(Acc)) / 16;
  static_assert(QN * 16 == V * static_cast<int>(sizeof(Acc)), "partial vector size");
  union PartialVec {
    uint4 q[QN];
    Acc a[V];
  };
  if (ph == 0 && has) {
    PartialVec u;
#pragma unroll
    for (int i = 0; i < V; ++i) u.a[i] = acc[i];
    uint4* dst = reinterpret_cast<uint4*>(partials + static_cast<int64_t>(blockIdx.y) * M + col);
#pragma unroll
    for (int q = 0; q < QN; ++q) __stcg(dst + q, u.q[q]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&counters[blockIdx.x], 1u);
    if (prev >= splits) record_device_error(kDevErrSplitReduce);
    s_last = (prev == splits - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Thread (cv, ph) adds splits ph, ph + P, ... in ascending order, loads
  // issued GS_T_RED_BATCH at a time; then the phases are added in order.
  Acc sum[V];
#pragma unroll
  for (int i = 0; i < V; ++i) sum[i] = 0;
  if (has) {
    constexpr int GS_T_RED_BATCH = GS_T_RED_REGS / (V * static_cast<int>(sizeof(Acc)) / 4);
    for (unsigned int k0 = ph; k0 < splits; k0 += GS_T_RED_BATCH * P) {
      Acc pv[GS_T_RED_BATCH][V];
#pragma unroll
      for (int b = 0; b < GS_T_RED_BATCH; ++b) {
        const unsigned int k = k0 + b * P;
        PartialVec u;
        const uint4* src = reinterpret_cast<const uint4*>(partials + static_cast<int64_t>(k) * M + col);
#pragma unroll
        for (int q = 0; q < QN; ++q) u.q[q] = (k < splits) ? __ldcg(src + q) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < V; ++i) pv[b][i] = u.a[i];
      }
#pragma unroll
      for (int b = 0; b < GS_T_RED_BATCH; ++b)
        if (k0 + b * P < splits)
#pragma unroll
          for (int i = 0; i < V; ++i) sum[i] += pv[b][i];
    }
  }
  if (ph > 0) {
#pragma unroll
    for (int i = 0; i < V; ++i) s_phase[ph - 1][cv * V + i] = sum[i];
  }
  __syncthreads();
  if (ph == 0 && has) {
#pragma unroll
    for (int q = 0; q < P - 1; ++q)
#pragma unroll
      for (int i = 0; i < V; ++i) sum[i] += s_phase[q][cv * V + i];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      y[col + i] =
          from_acc<T>(beta != Acc(0) ? epi_axpby(alpha, sum[i], beta, to_acc<T>(y[col + i])) : epi_scale(alpha, sum[i]));
    }
  }
  if (tid == 0) counters[blockIdx.x] = 0u;
}

}  // namespace

struct GemvStreamPlan {
  bool ok = false;
  bool trans = false;
  int kv = 0;                 // gemv_n_xreg vectors per lane
  int64_t grid = 0;           // gemv_n_xreg CTAs
  int rows_per_cta = 0;
  int64_t strips = 0, splits = 0, rows_per_split = 0;  // gemv_t_lsu
  size_t partial_bytes = 0;
};

template <typename T>
GemvStreamPlan plan_gemv_stream(int trans, int64_t M, int64_t N, int64_t lda, const void* A, const void* x,
                                int sms) {
  GemvStreamPlan p;
  using Acc = typename AccOf<T>::type;
  constexpr int V = 16 / sizeof(T);
  const bool a_al = (reinterpret_cast<uintptr_t>(A) % 16 == 0) && ((lda * (int64_t)sizeof(T)) % 16 == 0);
  if (!a_al || M <= 0 || N <= 0) return p;
  const int64_t ctas_full = 2LL * sms;  // two resident CTAs per SM
  if (!trans) {
    if (N % V || reinterpret_cast<uintptr_t>(x) % 16) return p;
    const int64_t nvec = N / V;
    if (nvec > 8 * 32 * GS_WARPS) return p;  // x slice must fit 8 vectors per lane
    if (M < sms) return p;                    // short-wide shapes: split-K kernel
    int kv = 1;
    while (kv * 32 * GS_WARPS < nvec) kv *= 2;
    p.kv = kv;
    // Two waves of CTAs: a CTA that finishes early picks up a second row
    // block, which evens out per-SM bandwidth differences at the tail.
    int64_t rows = (M + 2 * ctas_full - 1) / (2 * ctas_full);
    rows = std::min<int64_t>(std::max<int64_t>(rows, 1), GS_ROWS_MAX);
    p.rows_per_cta = static_cast<int>(rows);
    p.grid = (M + rows - 1) / rows;
    p.ok = true;
  } else {
    if (M % V || N < 16) return p;
    const int64_t strip = static_cast<int64_t>(GS_T_SV) * V;
    p.strips = (M + strip - 1) / strip;
    if (p.strips > 4096) return p;
    // Whole batches of GS_T_UNROLL rows per phase in each split (only the
    // last split may end in a partial batch).
    const int64_t batch_rows = static_cast<int64_t>(GS_T_UNROLL) * GS_T_PHASES;
    int64_t splits = std::max<int64_t>(1, GS_T_WAVES * ctas_full / p.strips);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, N / batch_rows));
    splits = std::min<int64_t>(splits, 65535);
    p.rows_per_split = ((N + splits - 1) / splits + batch_rows - 1) / batch_rows * batch_rows;
    p.splits = (N + p.rows_per_split - 1) / p.rows_per_split;
    if (p.splits > 1) p.partial_bytes = (static_cast<size_t>(p.splits) * M * sizeof(Acc) + 255) / 256 * 256;
    p.trans = true;
    p.ok = true;
  }
  return p;
}

// Returns -1 when these kernels do not apply (caller falls back), else a
// status.  Workspace layout matches gemv.cu: [counters][partials].
template <typename T>
int launch_gemv_stream(int trans, int64_t M, int64_t N, double alpha_d, const void* A_, int64_t lda,
                       const void* x_, double beta_d, void* y_, void* ws, size_t ws_bytes, size_t counter_bytes,
                       cudaStream_t stream) {
  using Acc = typename AccOf<T>::type;
  const int sms = device_sm_count();
  const GemvStreamPlan p = plan_gemv_stream<T>(trans, M, N, lda, A_, x_, sms);
  if (!p.ok) return -1;
  if (p.trans && p.splits > 1 &&
      (ws == nullptr || ws_bytes < counter_bytes + p.partial_bytes || reinterpret_cast<uintptr_t>(ws) % 256))
    return -1;
  const T* A = static_cast<const T*>(A_);
  const T* x = static_cast<const T*>(x_);
  T* y = static_cast<T*>(y_);
  const Acc alpha = static_cast<Acc>(alpha_d), beta = static_cast<Acc>(beta_d);
  if (!p.trans) {
    const dim3 grid(static_cast<unsigned>(p.grid));
    cudaError_t e;
    const int rpc = p.rows_per_cta;
    switch (p.kv) {
      case 1: e = launch_pdl(gemv_n_xreg<T, 1>, grid, dim3(GS_THREADS), 0, stream, M, N, alpha, A, lda, x, beta, y, rpc); break;
      case 2: e = launch_pdl(gemv_n_xreg<T, 2>, grid, dim3(GS_THREADS), 0, stream, M, N, alpha, A, lda, x, beta, y, rpc); break;
      case 4: e = launch_pdl(gemv_n_xreg<T, 4>, grid, dim3(GS_THREADS), 0, stream, M, N, alpha, A, lda, x, beta, y, rpc); break;
      default: e = launch_pdl(gemv_n_xreg<T, 8>, grid, dim3(GS_THREADS), 0, stream, M, N, alpha, A, lda, x, beta, y, rpc); break;
    }
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_failure(e);
    }
    note_launch("gemv_n_xreg");
  } else {
    unsigned int* counters = reinterpret_cast<unsigned int*>(ws);
    Acc* partials = reinterpret_cast<Acc*>(static_cast<char*>(ws) + counter_bytes);
    const dim3 grid(static_cast<unsigned>(p.strips), static_cast<unsigned>(p.splits));
    const cudaError_t e = launch_pdl(gemv_t_lsu<T>, grid, dim3(GS_THREADS), 0, stream, M, N, alpha, A, lda, x, beta,
                                     y, p.rows_per_split, partials, counters);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return cuda_failure(e);
    }
    note_launch("gemv_t_lsu");
  }
  return check_launch();
}

size_t gemv_stream_workspace(int dtype, int trans, int64_t M, int64_t N) {
  const void* al = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  const int sms = device_sm_count();
  GemvStreamPlan p;
  const int64_t lda = trans ? M : N;
  switch (dtype) {
    case CUOPX_F32: p = plan_gemv_stream<float>(trans, M, N, lda, al, al, sms); break;
    case CUOPX_F64: p = plan_gemv_stream<double>(trans, M, N, lda, al, al, sms); break;
    case CUOPX_F16: p = plan_gemv_stream<__half>(trans, M, N, lda, al, al, sms); break;
    case CUOPX_BF16: p = plan_gemv_stream<__nv_bfloat16>(trans, M, N, lda, al, al, sms); break;
    default: return 0;
  }
  return p.ok ? p.partial_bytes : 0;
}

}  // namespace cuopx
