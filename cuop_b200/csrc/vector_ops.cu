// Level-1 vector operations (fp32) and the column-block gather used after an
// all-gather of N-sharded GEMM outputs.
//
// The reference's vector-ops plugin (src/jit/Blas/vector_ops_jit_plugin.cu:317-665)
// defines DOT/AXPY/SCAL/COPY/SWAP/ROT/NRM2/ASUM/IAMAX/IAMIN; this file
// implements the standard BLAS meaning of each (nrm2 = sqrt(sum x^2) computed
// once, i?amax/i?amin = first 1-based index of the extreme |x_i|), which is
// what the plugin's kernels were written to compute.  Reductions are
// grid-stride partial sums per CTA followed by a last-arriving-CTA pass in
// fixed CTA order, so results are deterministic run to run.
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int VT = 256;        // threads per CTA
constexpr int MAX_RED_CTAS = 1024;

__device__ __forceinline__ int64_t vidx(int64_t i, int64_t n, int64_t inc) {
  return inc >= 0 ? i * inc : (n - 1 - i) * (-inc);
}

// ---------------------------------------------------------------- elementwise
__global__ void axpy_kernel(int64_t n, float alpha, const float* __restrict__ x, int64_t incx,
                            float* __restrict__ y, int64_t incy) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float* py = y + vidx(i, n, incy);
    *py = fmaf(alpha, x[vidx(i, n, incx)], *py);
  }
}

__global__ void scal_kernel(int64_t n, float alpha, float* __restrict__ x, int64_t incx) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float* px = x + vidx(i, n, incx);
    *px = alpha * *px;
  }
}

__global__ void copy_kernel(int64_t n, const float* __restrict__ x, int64_t incx, float* __restrict__ y,
                            int64_t incy) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[vidx(i, n, incy)] = x[vidx(i, n, incx)];
}

__global__ void swap_kernel(int64_t n, float* __restrict__ x, int64_t incx, float* __restrict__ y, int64_t incy) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float* px = x + vidx(i, n, incx);
    float* py = y + vidx(i, n, incy);
    const float t = *px;
    *px = *py;
    *py = t;
  }
}

__global__ void rot_kernel(int64_t n, float* __restrict__ x, int64_t incx, float* __restrict__ y, int64_t incy,
                           float c, float s) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float* px = x + vidx(i, n, incx);
    float* py = y + vidx(i, n, incy);
    const float xv = *px, yv = *py;
    *px = c * xv + s * yv;
    *py = c * yv - s * xv;
  }
}

// ---------------------------------------------------------------- reductions
enum RedOp { kDot = 0, kAsum = 1, kNrm2 = 2, kIamax = 3, kIamin = 4 };

struct Workspace {
  double* partial;        // [MAX_RED_CTAS]
  int64_t* index;         // [MAX_RED_CTAS]
  unsigned int* counter;  // [1]
};

__device__ __forceinline__ bool better(int op, double v, int64_t i, double bv, int64_t bi) {
  if (bi < 0) return true;
  if (op == kIamax) return v > bv || (v == bv && i < bi);
  return v < bv || (v == bv && i < bi);
}

template <int OP>
__global__ void __launch_bounds__(VT) reduce_kernel(int64_t n, const float* __restrict__ x, int64_t incx,
                                                    const float* __restrict__ y, int64_t incy, Workspace ws,
                                                    float* __restrict__ fres, int64_t* __restrict__ ires) {
  __shared__ double s_val[VT];
  __shared__ int64_t s_idx[VT];
  __shared__ unsigned int s_last;
  double acc = 0.0;
  int64_t bi = -1;
  for (int64_t i = blockIdx.x * (int64_t)VT + threadIdx.x; i < n; i += (int64_t)gridDim.x * VT) {
    const float xv = x[vidx(i, n, incx)];
    if (OP == kDot) acc += static_cast<double>(xv) * static_cast<double>(y[vidx(i, n, incy)]);
    if (OP == kAsum) acc += fabs(static_cast<double>(xv));
    if (OP == kNrm2) acc += static_cast<double>(xv) * static_cast<double>(xv);
    if (OP == kIamax || OP == kIamin) {
      const double a = fabs(static_cast<double>(xv));
      if (better(OP, a, i, acc, bi)) acc = a, bi = i;
    }
  }
  s_val[threadIdx.x] = acc;
  s_idx[threadIdx.x] = bi;
  __syncthreads();
  for (int w = VT / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      if (OP == kIamax || OP == kIamin) {
        const int o = threadIdx.x + w;
        if (s_idx[o] >= 0 && better(OP, s_val[o], s_idx[o], s_val[threadIdx.x], s_idx[threadIdx.x])) {
          s_val[threadIdx.x] = s_val[o];
          s_idx[threadIdx.x] = s_idx[o];
        }
      } else {
        s_val[threadIdx.x] += s_val[threadIdx.x + w];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ws.partial[blockIdx.x] = s_val[0];
    ws.index[blockIdx.x] = s_idx[0];
    __threadfence();
    const unsigned int prev = atomicAdd(ws.counter, 1u);
    if (prev >= gridDim.x) record_device_error(kDevErrSplitReduce);
    s_last = (prev == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  double tot = 0.0;
  int64_t tidx = -1;
  for (unsigned int b = 0; b < gridDim.x; ++b) {
    const double v = __ldcg(&ws.partial[b]);
    const int64_t ix = __ldcg(&ws.index[b]);
    if (OP == kIamax || OP == kIamin) {
      if (ix >= 0 && better(OP, v, ix, tot, tidx)) tot = v, tidx = ix;
    } else {
      tot += v;
    }
  }
  if (OP == kDot || OP == kAsum) *fres = static_cast<float>(tot);
  if (OP == kNrm2) *fres = static_cast<float>(sqrt(tot));
  if (OP == kIamax || OP == kIamin) *ires = tidx + 1;  // 1-based; 0 when n == 0
  *ws.counter = 0u;
}

int grid_for(int64_t n) {
  const int64_t want = (n + VT * 4 - 1) / (VT * 4);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, device_sm_count() * 8)));
}

// ---------------------------------------------------------------- gather
// blocks: [G][M][Nb] -> out[M][ldo] with out[m][g*Nb + j] = blocks[g][m][j].
template <typename T>
__global__ void gather_kernel(int64_t G, int64_t M, int64_t Nb, const T* __restrict__ blocks, T* __restrict__ out,
                              int64_t ldo) {
  const int64_t total = G * M * Nb;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e % Nb;
    const int64_t m = (e / Nb) % M;
    const int64_t g = e / (Nb * M);
    out[m * ldo + g * Nb + j] = blocks[e];
  }
}

}  // namespace

size_t vector_workspace_size_impl() {
  return static_cast<size_t>(MAX_RED_CTAS) * (sizeof(double) + sizeof(int64_t)) + 256;
}

int vector_reduce(int op, int64_t n, const float* x, int64_t incx, const float* y, int64_t incy, float* fres,
                  int64_t* ires, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (!workspace || ws_bytes < vector_workspace_size_impl() || (reinterpret_cast<uintptr_t>(workspace) % 16))
    return CUOPX_INVALID_ARGUMENT;
  Workspace ws;
  ws.partial = static_cast<double*>(workspace);
  ws.index = reinterpret_cast<int64_t*>(static_cast<char*>(workspace) + MAX_RED_CTAS * sizeof(double));
  ws.counter = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) +
                                               MAX_RED_CTAS * (sizeof(double) + sizeof(int64_t)));
  const int grid = std::min(grid_for(n), MAX_RED_CTAS);
  switch (op) {
    case kDot: reduce_kernel<kDot><<<grid, VT, 0, stream>>>(n, x, incx, y, incy, ws, fres, ires); break;
    case kAsum: reduce_kernel<kAsum><<<grid, VT, 0, stream>>>(n, x, incx, y, incy, ws, fres, ires); break;
    case kNrm2: reduce_kernel<kNrm2><<<grid, VT, 0, stream>>>(n, x, incx, y, incy, ws, fres, ires); break;
    case kIamax: reduce_kernel<kIamax><<<grid, VT, 0, stream>>>(n, x, incx, y, incy, ws, fres, ires); break;
    case kIamin: reduce_kernel<kIamin><<<grid, VT, 0, stream>>>(n, x, incx, y, incy, ws, fres, ires); break;
    default: return CUOPX_INVALID_ARGUMENT;
  }
  static const char* names[] = {"vec_dot", "vec_asum", "vec_nrm2", "vec_iamax", "vec_iamin"};
  note_launch(names[op]);
  return check_launch();
}

int vector_elementwise(int op, int64_t n, float alpha, const float* x, int64_t incx, float* y, int64_t incy,
                       float c, float s, float* xm, cudaStream_t stream) {
  const int grid = grid_for(n);
  switch (op) {
    case 0: axpy_kernel<<<grid, VT, 0, stream>>>(n, alpha, x, incx, y, incy); note_launch("vec_axpy"); break;
    case 1: scal_kernel<<<grid, VT, 0, stream>>>(n, alpha, xm, incx); note_launch("vec_scal"); break;
    case 2: copy_kernel<<<grid, VT, 0, stream>>>(n, x, incx, y, incy); note_launch("vec_copy"); break;
    case 3: swap_kernel<<<grid, VT, 0, stream>>>(n, xm, incx, y, incy); note_launch("vec_swap"); break;
    case 4: rot_kernel<<<grid, VT, 0, stream>>>(n, xm, incx, y, incy, c, s); note_launch("vec_rot"); break;
    default: return CUOPX_INVALID_ARGUMENT;
  }
  return check_launch();
}

int gather_column_blocks(int dtype, int64_t G, int64_t M, int64_t Nb, const void* blocks, void* out, int64_t ldo,
                         cudaStream_t stream) {
  const int64_t total = G * M * Nb;
  if (total == 0) return CUOPX_SUCCESS;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, device_sm_count() * 16));
  switch (dtype_size(dtype)) {
    case 2:
      gather_kernel<uint16_t><<<grid, 256, 0, stream>>>(G, M, Nb, static_cast<const uint16_t*>(blocks),
                                                        static_cast<uint16_t*>(out), ldo);
      break;
    case 4:
      gather_kernel<uint32_t><<<grid, 256, 0, stream>>>(G, M, Nb, static_cast<const uint32_t*>(blocks),
                                                        static_cast<uint32_t*>(out), ldo);
      break;
    case 8:
      gather_kernel<uint64_t><<<grid, 256, 0, stream>>>(G, M, Nb, static_cast<const uint64_t*>(blocks),
                                                        static_cast<uint64_t*>(out), ldo);
      break;
    default: return CUOPX_UNSUPPORTED_TYPE;
  }
  note_launch("gather_column_blocks");
  return check_launch();
}

}  // namespace cuopx
