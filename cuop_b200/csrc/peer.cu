// Peer memory, the cross-GPU barrier and the fused column-sharded GEMM +
// all-gather (cuopx_gemm_allgather).  One process per GPU; peers are the
// other GPUs of the node, reached over NVLink/NVSwitch through CUDA IPC
// mappings.  The reference is single-GPU and has no counterpart.
//
// Ordering contract of cuopx_peer_barrier: each rank's stream runs
//   [writes, possibly to peers] -> barrier kernel -> [reads]
// The barrier kernel issues a system-scope fence, posts its epoch into every
// rank's signal block with st.release.sys, then spins (ld.acquire.sys, at
// most kPeerWaitLimitNs) until every rank has posted the same epoch into its
// own block.  Kernel boundaries on a stream order the earlier writes before
// the fence, so after the barrier every rank sees every rank's writes.
#include <cstring>

#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int kMaxRanks = 8;
// Slots [0, kMaxRanks) of a signal block: epoch posted by rank r.  The local
// epoch counter sits in its own 128-byte line.
constexpr int kEpochSlot = 64;
// Peers can be late by host-side skew (first-call set-up on another rank),
// so this wait is longer than the in-kernel pipeline waits.
constexpr unsigned long long kPeerWaitLimitNs = 5ull * 1000ull * 1000ull * 1000ull;

static_assert(sizeof(cudaIpcMemHandle_t) == CUOPX_PEER_HANDLE_BYTES, "IPC handle size");
static_assert((kEpochSlot + 1) * 4 <= CUOPX_PEER_SIGNAL_BYTES, "signal block layout");
static_assert(kDevErrPeerTimeout == CUOPX_DEVERR_PEER_TIMEOUT, "device error code");

struct SignalPtrs {
  unsigned int* p[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(unsigned int* addr, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* addr) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(SignalPtrs s, int world, int rank) {
  const int t = threadIdx.x;
  unsigned int* mine = s.p[rank];
  unsigned int e = 0;
  if (t == 0) {
    e = mine[kEpochSlot] + 1u;
    mine[kEpochSlot] = e;
  }
  e = __shfl_sync(0xffffffffu, e, 0);
  __threadfence_system();
  if (t < world) st_release_sys(s.p[t] + rank, e);
  if (t < world) {
    const unsigned long long t0 = global_timer_ns();
    while (static_cast<int>(ld_acquire_sys(mine + t) - e) < 0) {
      if (global_timer_ns() - t0 > kPeerWaitLimitNs) {
        record_device_error(kDevErrPeerTimeout);
        break;
      }
    }
  }
  __syncwarp();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

}  // namespace cuopx

using namespace cuopx;

extern "C" {

int cuopx_peer_alloc(size_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes == 0) return CUOPX_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return CUOPX_OUT_OF_MEMORY;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return CUOPX_CUDA_ERROR;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return CUOPX_SUCCESS;
}

int cuopx_peer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return CUOPX_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return CUOPX_CUDA_ERROR;
  }
  *ptr = p;
  return CUOPX_SUCCESS;
}

int cuopx_peer_close(void* ptr) {
  if (!ptr) return CUOPX_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? CUOPX_SUCCESS : CUOPX_CUDA_ERROR;
}

int cuopx_peer_free(void* ptr) {
  if (!ptr) return CUOPX_INVALID_ARGUMENT;
  return cudaFree(ptr) == cudaSuccess ? CUOPX_SUCCESS : CUOPX_CUDA_ERROR;
}

int cuopx_peer_barrier(void* const* signals, int world, int rank, void* stream) {
  if (!signals || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return CUOPX_INVALID_ARGUMENT;
  SignalPtrs s{};
  for (int r = 0; r < world; ++r) {
    if (!signals[r] || !aligned16(signals[r])) return CUOPX_INVALID_ARGUMENT;
    s.p[r] = static_cast<unsigned int*>(signals[r]);
  }
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(s, world, rank);
  note_launch("peer_barrier");
  return check_launch();
}

int cuopx_gemm_allgather(int dtype, int transA, int transB, int64_t M, int64_t N_local, int64_t K, double alpha,
                         const void* A, int64_t lda, const void* B, int64_t ldb, void* const* C_ranks, int world,
                         int rank, int64_t ldc, void* stream) {
  if (dtype_size(dtype) == 0) return CUOPX_UNSUPPORTED_TYPE;
  if (!C_ranks || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return CUOPX_INVALID_ARGUMENT;
  if (M < 0 || N_local < 0 || K < 0) return CUOPX_INVALID_ARGUMENT;
  if (ldc < world * N_local) return CUOPX_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (!C_ranks[r]) return CUOPX_INVALID_ARGUMENT;
  if (M == 0 || N_local == 0) return CUOPX_SUCCESS;
  if (dtype != CUOPX_F16 && dtype != CUOPX_BF16) return CUOPX_NOT_IMPLEMENTED;
  if (M < 256 || N_local < 256 || K < 256 || N_local % 8 != 0 || ldc % 8 != 0) return CUOPX_NOT_IMPLEMENTED;
  const size_t es = dtype_size(dtype);
  GemmProblem p{};
  p.dtype = dtype;
  p.transA = transA != 0;
  p.transB = transB != 0;
  p.M = M;
  p.N = N_local;
  p.K = K;
  p.alpha = alpha;
  p.beta = 0.0;
  p.A = A;
  p.lda = lda;
  p.B = B;
  p.ldb = ldb;
  p.C = static_cast<unsigned char*>(C_ranks[rank]) + static_cast<size_t>(rank) * N_local * es;
  p.ldc = ldc;
  p.batch = 1;
  p.strideA = p.strideB = p.strideC = 0;
  const int rc = validate_gemm(p);
  if (rc >= 0) return rc;
  if (!gemm_tc_supported(p)) return CUOPX_NOT_IMPLEMENTED;
  void* peers[kMaxRanks - 1];
  int np = 0;
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    if (!aligned16(C_ranks[r])) return CUOPX_INVALID_ARGUMENT;
    peers[np++] = static_cast<unsigned char*>(C_ranks[r]) + static_cast<size_t>(rank) * N_local * es;
  }
  // Tile choice: 2-SM pair tiles at every rank count.  Measured on B200 at
  // 8 ranks (same box, same inputs), pair tiles beat the 1-SM peer paths
  // even where the exchange outlasts the GEMM (C3 8192^3: 271 us vs 285 us
  // for 128 x 256 and 305 us for 128 x 128 tiles; C5: 401 vs 428 / 450 us).
  // The pair tile width follows the block's size (256 x 512 tiles when
  // there are two waves of them).  A variant override
  // (cuopx_set_gemm_variant[_thread]) selects a width or a 1-SM path.
  const int v = select_gemm_variant(p);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v == kVariantTc128x256) return gemm_tc_peers(p, peers, np, s, 256);
  if (v == kVariantTc128x128) return gemm_tc_peers(p, peers, np, s, 128);
  if (v == kVariantTc2) return gemm_tc2_peers(p, peers, np, s, 256);
  if (v == kVariantTc2x512) return gemm_tc2_peers(p, peers, np, s, 512);
  if (v == kVariantTc2x128) return gemm_tc2_peers(p, peers, np, s, 128);
  return gemm_tc2_peers(p, peers, np, s);
}

}  // extern "C"
