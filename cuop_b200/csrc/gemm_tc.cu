// tcgen05 / TMEM / TMA GEMM for fp16 and bf16 inputs (fp32 accumulate),
// plain and strided-batched, any transpose combination.
//
// The grid has one CTA per output tile, but a CTA does not stop after its
// own tile: before finishing a tile it asks the hardware (cluster launch
// control, clusterlaunchcontrol.try_cancel) to cancel a CTA that has not been
// launched yet and takes over that CTA's tile.  The first wave of CTAs (one
// per SM) therefore runs persistently, and an SM that is fast takes more
// tiles than one that is slow, with no tile counter in global memory.
// Every role of the CTA reads the same responses from a shared-memory ring,
// so producer, MMA issuer and epilogue walk the same tile sequence.
// 6 warps, warp-specialised:
//   warp 0      TMA producer: K-blocks of A (128 x 64) and B (BN x 64) into a
//               STAGES-deep shared-memory ring (128-byte swizzle), one
//               mbarrier pair (full/empty) per stage.
//   warp 1      TMEM allocator + MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) into a
//               TMEM accumulator; tcgen05.commit frees smem stages and hands
//               finished accumulators to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld (32 lanes x 32 columns), alpha/beta in
//               fp32, one rounding to the output type, 128-byte-swizzled
//               staging in smem, TMA bulk tensor store.
// The accumulator is double (BN=256) or quadruple (BN=128) buffered in the
// 512 TMEM columns so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Semantics: C = alpha * op(A) op(B) + beta * C (the reference's Gemm<T>
// contract, src/cuda_op/detail/cuBlas/gemm.cu:41, batched form
// src/jit/Blas/gemm_batched_jit_plugin.cu:324-330) with fp16/bf16 inputs,
// fp32 products and sums, result rounded once (round-to-nearest-even).
//
// No TMA multicast is used anywhere in this file.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes = one swizzle row
constexpr int NUM_THREADS = 192;
constexpr int EPI_WARPS = 4;
constexpr int STAGE_CHUNK_COLS = 64;  // epilogue column chunk (one TMA store box)
constexpr int GROUP_M = 16;  // raster: walk 16 M-tiles per N step for L2 reuse
constexpr bool TC_PREFETCH_FIRST_TILE = true;
// Scheduler ring depth: more than the producer's lead over the epilogue
// (STAGES + accumulator buffers, in tiles), so the producer never waits on it.
constexpr int CLC_SLOTS = 16;
// Arrivals that free a scheduler slot: producer, MMA issuer, epilogue warps.
constexpr int CLC_READERS = 2 + EPI_WARPS;

struct TcParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, num_tiles, k_blocks;
  float alpha, beta;
  const void* C_in;  // read only when beta != 0
  int64_t ldc, strideC;
  const void* bias;  // CUOPX_EPI_BIAS: N elements of the output type
  int epi;           // CUOPX_EPI_* flags
  // Peer-store all-gather: each staged output chunk is also written to
  // peer_C[i] (same row stride ldc, same column offset) for i < npeers.
  int npeers;
  void* peer_C[7];
  // L2 prefetch before the dependent-launch wait: a CTA with blockIdx.x <
  // wave (the first wave) warms the K blocks of tiles blockIdx.x + j * wave,
  // j < prefetch_tiles (up to STAGES K blocks each); others only their own.
  int wave, prefetch_tiles;
};

// CPS: CTAs resident per SM (1, or 2 for short-K problems: two CTAs of this
// kernel, or one of it and one of the next launch, share the SM); each CTA
// owns 512 / CPS TMEM columns.
template <int BN, int STAGES, int CPS = 1>
struct SmemLayout {
  static constexpr uint32_t TMEM_COLS = 512u / CPS;
  static constexpr int A_STAGE = BM * BK * 2;
  static constexpr int B_STAGE = BN * BK * 2;
  static constexpr int C_STAGE = 32 * STAGE_CHUNK_COLS * 2;  // one warp's staging buffer
  static constexpr int ACC_BUFS = TMEM_COLS / BN;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE;
  static constexpr int OFF_C = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_BAR = OFF_C + EPI_WARPS * 2 * C_STAGE;
  // full[STAGES], empty[STAGES], acc_full[ACC_BUFS], acc_empty[ACC_BUFS], drain
  static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 1;
  // Tile-scheduler ring: CLC_SLOTS 16-byte launch-control responses, then
  // clc_full[CLC_SLOTS] and clc_empty[CLC_SLOTS] mbarriers.
  static constexpr int OFF_CLC = (OFF_BAR + NUM_BARS * 8 + 15) / 16 * 16;
  static constexpr int OFF_CLC_BAR = OFF_CLC + CLC_SLOTS * 16;
  static constexpr int OFF_MISC = OFF_CLC_BAR + 2 * CLC_SLOTS * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;  // slack for 1024-byte alignment
  static_assert(ALLOC <= 232448, "shared memory budget exceeded");
  static_assert(CPS == 1 || (ALLOC + 1024) * CPS <= 233472, "CPS CTAs must fit one SM's shared memory");
  static_assert(ACC_BUFS >= 2, "the epilogue overlaps the next tile's MMAs");
};

__device__ __forceinline__ void tile_coords(int t, const TcParams& p, int& b, int& mt, int& nt) {
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;
  const int r = t - b * per_batch;
  const int span = GROUP_M * p.tiles_n;
  const int g = r / span;
  const int first_m = g * GROUP_M;
  const int gsize = min(GROUP_M, p.tiles_m - first_m);
  const int rr = r - g * span;
  mt = first_m + rr % gsize;
  nt = rr / gsize;
}

// Next tile from a completed launch-control response; false when the grid
// has no unlaunched CTA left (or, defensively, the answer is out of range).
__device__ __forceinline__ bool clc_next_tile(const void* resp, int num_tiles, int& next) {
  if (!clc_query(resp, next)) return false;
  if (next < 0 || next >= num_tiles) {
    record_device_error(kDevErrSchedule);
    return false;
  }
  return true;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, int BN, int STAGES, bool A_MN, bool B_MN, bool PEERS = false, int CPS = 1>
__global__ void __launch_bounds__(NUM_THREADS, CPS)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using L = SmemLayout<BN, STAGES, CPS>;
  constexpr uint32_t TMEM_COLS = L::TMEM_COLS;
  constexpr int ACC_BUFS = L::ACC_BUFS;
  constexpr uint32_t STAGE_TX = static_cast<uint32_t>(L::A_STAGE + L::B_STAGE);
  constexpr uint32_t AB_FMT = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t IDESC = make_idesc(AB_FMT, A_MN, B_MN, BM, BN);

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = align_smem_1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + ACC_BUFS;
  uint64_t* drain = bars + 2 * STAGES + 2 * ACC_BUFS;
  unsigned char* clc_resp = smem + L::OFF_CLC;
  uint64_t* clc_full = reinterpret_cast<uint64_t*>(smem + L::OFF_CLC_BAR);
  uint64_t* clc_empty = clc_full + CLC_SLOTS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ACC_BUFS; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], EPI_WARPS);
    }
    for (int c = 0; c < CLC_SLOTS; ++c) {
      mbar_init(&clc_full[c], 1);
      mbar_init(&clc_empty[c], CLC_READERS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
    if (TC_PREFETCH_FIRST_TILE) {
      // L2 prefetch while the previous kernel on the stream may still be
      // draining: this CTA's first tile and, for a first-wave CTA, the tiles
      // the grid runs after the first wave (up to STAGES K blocks each).  It
      // only warms L2, the device's point of coherence, so it cannot return
      // data older than the previous kernel's writes; every load stays after
      // the dependent-launch wait.
      const int tiles_ahead = static_cast<int>(blockIdx.x) < p.wave ? p.prefetch_tiles : 1;
      for (int j = 0; j < tiles_ahead; ++j) {
        const int64_t t = static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(j) * p.wave;
        if (t >= p.num_tiles) break;
        int b, mt, nt;
        tile_coords(static_cast<int>(t), p, b, mt, nt);
        const int m0 = mt * BM, n0 = nt * BN;
        for (int kb = 0; kb < min(p.k_blocks, STAGES); ++kb) {
          const int k0 = kb * BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int jj = 0; jj < BM / 64; ++jj) tma_prefetch_3d(&tmA, m0 + 64 * jj, k0, b);
          } else {
            tma_prefetch_3d(&tmA, k0, m0, b);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int jj = 0; jj < BN / 64; ++jj) tma_prefetch_3d(&tmB, n0 + 64 * jj, k0, b);
          } else {
            tma_prefetch_3d(&tmB, k0, n0, b);
          }
        }
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touched only shared memory, TMEM and the parameter
  // tensor maps; global memory waits for the previous kernel on the stream.
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // Abort bookkeeping, one bit per stage: loaded at least once, and the
      // parity of the last phase loaded.
      uint32_t issued_mask = 0, phase_mask = 0;
      bool ok = true;
      bool clc_pending = false;
      int cs = 0;
      uint32_t cpar = 0;
      int t = blockIdx.x;
      for (int seq = 0; ok; ++seq) {
        // Ask for the tile after this one now, so the answer is in by the
        // time this tile's loads are issued.
        cs = seq % CLC_SLOTS;
        cpar = static_cast<uint32_t>(seq / CLC_SLOTS) & 1u;
        if (!mbar_wait_bounded(&clc_empty[cs], cpar ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&clc_full[cs], 16);
        clc_try_cancel(clc_resp + cs * 16, &clc_full[cs]);
        clc_pending = true;
        int b, mt, nt;
        tile_coords(t, p, b, mt, nt);
        const int m0 = mt * BM, n0 = nt * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          unsigned char* sa = smem + L::OFF_A + stage * L::A_STAGE;
          unsigned char* sb = smem + L::OFF_B + stage * L::B_STAGE;
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          const int k0 = kb * BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_3d(sa + j * (64 * BK * 2), &tmA, &full[stage], m0 + 64 * j, k0, b);
          } else {
            tma_load_3d(sa, &tmA, &full[stage], k0, m0, b);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(sb + j * (64 * BK * 2), &tmB, &full[stage], n0 + 64 * j, k0, b);
          } else {
            tma_load_3d(sb, &tmB, &full[stage], k0, n0, b);
          }
          issued_mask |= 1u << stage;
          phase_mask = (phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        if (!mbar_wait_bounded(&clc_full[cs], cpar, kDevErrWaitTimeoutFull, abort_flag)) {
          ok = false;
          break;
        }
        clc_pending = false;
        int next = 0;
        const bool more = clc_next_tile(clc_resp + cs * 16, p.num_tiles, next);
        mbar_arrive(&clc_empty[cs]);
        if (!more) {
          grid_launch_dependents();  // all loads issued: the next kernel may start its prologue
          break;
        }
        t = next;
      }
      if (!ok) {
        // Abort: let every load already issued, and the outstanding
        // launch-control response, land before the CTA exits.
        for (int s = 0; s < STAGES; ++s) {
          if (!((issued_mask >> s) & 1u)) continue;
          const uint32_t addr = smem_u32(&full[s]);
          const unsigned long long t0 = global_timer_ns();
          while (!mbar_try_wait(addr, (phase_mask >> s) & 1u)) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              record_device_error(kDevErrAbortDrain);
              break;
            }
          }
        }
        if (clc_pending) {
          const uint32_t addr = smem_u32(&clc_full[cs]);
          const unsigned long long t0 = global_timer_ns();
          while (!mbar_try_wait(addr, cpar)) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              record_device_error(kDevErrAbortDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int seq = 0; ok; ++seq) {
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, kDevErrWaitTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_u32(smem + L::OFF_A + stage * L::A_STAGE);
          const uint32_t sb = smem_u32(smem + L::OFF_B + stage * L::B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: advance 16 elements = 32 bytes inside the swizzled row.
            // MN-major: advance 16 rows of 128 bytes = 2048 bytes.
            const uint64_t ad = A_MN ? make_smem_desc_sw128(sa + kk * 2048, 64 * BK * 2, 1024)
                                     : make_smem_desc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                     : make_smem_desc_sw128(sb + kk * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty[stage]);  // stage is free once these MMAs have read it
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);  // accumulator complete
        if (++acc == ACC_BUFS) acc = 0, acc_phase ^= 1u;
        const int cs = seq % CLC_SLOTS;
        if (!mbar_wait_bounded(&clc_full[cs], static_cast<uint32_t>(seq / CLC_SLOTS) & 1u, kDevErrWaitTimeoutFull,
                               abort_flag))
          break;
        int next = 0;
        const bool more = clc_next_tile(clc_resp + cs * 16, p.num_tiles, next);
        mbar_arrive(&clc_empty[cs]);
        if (!more) break;
      }
      if (!ok && issued) {
        // Abort: make sure no MMA is still writing TMEM before dealloc.
        umma_commit(drain);
        const uint32_t addr = smem_u32(drain);
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(addr, 0)) {
          if (global_timer_ns() - t0 > kWaitLimitNs) {
            record_device_error(kDevErrAbortDrain);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = 32 * q + lane;
    unsigned char* const stage_base = smem + L::OFF_C + (warp - 2) * 2 * L::C_STAGE;  // two buffers
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    const T* Cin = static_cast<const T*>(p.C_in);
    int t = blockIdx.x;
    for (int seq = 0;; ++seq) {
      int b, mt, nt;
      tile_coords(t, p, b, mt, nt);
      const int m0 = mt * BM, n0 = nt * BN;
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, kDevErrWaitTimeoutAccFull, abort_flag)) break;
      tc_fence_after_sync();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(acc * BN);
      const int64_t grow = static_cast<int64_t>(m0) + row_in_tile;
#pragma unroll 1
      for (int ch = 0; ch < BN / STAGE_CHUNK_COLS; ++ch) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + ch * STAGE_CHUNK_COLS, r0);
        tmem_ld_32x32b_x32(t_row + ch * STAGE_CHUNK_COLS + 32, r1);
        tmem_wait_ld();
        if (ch == BN / STAGE_CHUNK_COLS - 1) {
          // Whole accumulator read: hand it back to the MMA warp.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        float v[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(r0[i]);
          v[32 + i] = __uint_as_float(r1[i]);
        }
        if (p.beta != 0.f && grow < p.M) {
          const int64_t gcol0 = static_cast<int64_t>(n0) + ch * STAGE_CHUNK_COLS;
          const T* crow = Cin + static_cast<int64_t>(b) * p.strideC + grow * p.ldc;
#pragma unroll
          for (int i = 0; i < 64; ++i)
            v[i] = gcol0 + i < p.N ? epi_axpby(p.alpha, v[i], p.beta, to_acc<T>(crow[gcol0 + i]))
                                   : epi_scale(p.alpha, v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] = epi_scale(p.alpha, v[i]);
        }
        if (p.epi) {
          const int64_t gcol0 = static_cast<int64_t>(n0) + ch * STAGE_CHUNK_COLS;
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (gcol0 + i < p.N) v[i] = apply_epilogue<T>(v[i], p.bias, gcol0 + i, p.epi);
        }
        // Stage 32 rows x 128 bytes, 128-byte swizzle (16-byte chunk j of row r at j ^ (r & 7)).
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        unsigned char* sbase = stage_base + sbuf * L::C_STAGE;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 w;
          w.x = pack2<T>(v[8 * j + 0], v[8 * j + 1]);
          w.y = pack2<T>(v[8 * j + 2], v[8 * j + 3]);
          w.z = pack2<T>(v[8 * j + 4], v[8 * j + 5]);
          w.w = pack2<T>(v[8 * j + 6], v[8 * j + 7]);
          *reinterpret_cast<uint4*>(sbase + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmC, sbase, n0 + ch * STAGE_CHUNK_COLS, m0 + 32 * q, b);
          bulk_commit_group();
        }
        if (PEERS && p.npeers > 0) {
          // Same 32 x 64 chunk to every peer's output: lanes 8r..8r+7 write
          // the 128 contiguous bytes of one row (four full 128-byte lines per
          // warp store).  Rows past M and 16-byte groups past N are skipped.
          const int c16 = lane & 7;
          const int64_t gcol = static_cast<int64_t>(n0) + ch * STAGE_CHUNK_COLS + 8 * c16;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (lane >> 3);
            const int64_t grow_r = static_cast<int64_t>(m0) + 32 * q + r;
            const uint4 w = *reinterpret_cast<const uint4*>(sbase + r * 128 + ((c16 ^ (r & 7)) << 4));
            if (grow_r < p.M && gcol < p.N) {
              const int64_t off = grow_r * p.ldc + gcol;
#pragma unroll
              for (int d = 0; d < 7; ++d)  // constant indices keep peer_C in the param bank
                if (d < p.npeers) *reinterpret_cast<uint4*>(static_cast<T*>(p.peer_C[d]) + off) = w;
            }
          }
        }
        sbuf ^= 1;
      }
      if (++acc == ACC_BUFS) acc = 0, acc_phase ^= 1u;
      const int cs = seq % CLC_SLOTS;
      if (!mbar_wait_bounded(&clc_full[cs], static_cast<uint32_t>(seq / CLC_SLOTS) & 1u, kDevErrWaitTimeoutAccFull,
                             abort_flag))
        break;
      int next = 0;
      const bool more = clc_next_tile(clc_resp + cs * 16, p.num_tiles, next);
      __syncwarp();
      if (lane == 0) mbar_arrive(&clc_empty[cs]);
      if (!more) break;
      t = next;
    }
    // Before the CTA exits, its shared memory must have been read by the
    // bulk stores; the stores themselves complete on their own and are
    // visible once the grid has completed (what the next kernel's
    // dependent-launch wait, or any later stream operation, waits for).
    // With peer outputs, the local stores are also waited for completely
    // before this thread's system-scope fence.
    if (lane == 0) {
      if (PEERS) bulk_wait_group<0>();
      else bulk_wait_group_read<0>();
    }
    __syncwarp();
    // Peer stores of this thread are ordered before anything the stream runs
    // after the kernel (the peer barrier's release).
    if (PEERS && p.npeers > 0) __threadfence_system();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D tiled map over a row-major [batch][rows][inner] tensor of `es`-byte
// elements with row stride `ld` and batch stride `bstride` (elements),
// 128-byte swizzle.
bool make_map_es(CUtensorMap* map, CUtensorMapDataType dt, int es, const void* base, int64_t inner, int64_t rows,
                 int64_t batch, int64_t ld, int64_t bstride, int box_inner, int box_rows,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = get_encode_fn();
  if (!enc) {
    cuda_failure_text("cuTensorMapEncodeTiled unavailable");
    return false;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * es),
                           static_cast<cuuint64_t>((batch > 1 ? bstride : ld * rows) * es)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) cuda_failure_text("cuTensorMapEncodeTiled failed");
  return r == CUDA_SUCCESS;
}

bool make_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int64_t inner, int64_t rows,
              int64_t batch, int64_t ld, int64_t bstride, int box_inner, int box_rows) {
  return make_map_es(map, dt, 2, base, inner, rows, batch, ld, bstride, box_inner, box_rows);
}

template <typename T, int BN, int STAGES, bool A_MN, bool B_MN, bool PEERS = false, int CPS = 1>
int launch_tc(const GemmProblem& p, cudaStream_t stream, const char* name, void* const* peers = nullptr,
              int npeers = 0) {
  using L = SmemLayout<BN, STAGES, CPS>;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mA, mB, mC;
  bool ok = true;
  // A: [K][M] when transposed (M contiguous) else [M][K].
  if (A_MN)
    ok &= make_map(&mA, dt, p.A, p.M, p.K, p.batch, p.lda, p.strideA, 64, BK);
  else
    ok &= make_map(&mA, dt, p.A, p.K, p.M, p.batch, p.lda, p.strideA, BK, BM);
  // B: [K][N] (N contiguous) when not transposed, else [N][K].
  if (B_MN)
    ok &= make_map(&mB, dt, p.B, p.N, p.K, p.batch, p.ldb, p.strideB, 64, BK);
  else
    ok &= make_map(&mB, dt, p.B, p.K, p.N, p.batch, p.ldb, p.strideB, BK, BN);
  ok &= make_map(&mC, dt, p.C, p.N, p.M, p.batch, p.ldc, p.strideC, STAGE_CHUNK_COLS, 32);
  if (!ok) return CUOPX_CUDA_ERROR;

  TcParams prm;
  prm.M = static_cast<int>(p.M);
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.tiles_m = static_cast<int>((p.M + BM - 1) / BM);
  prm.tiles_n = static_cast<int>((p.N + BN - 1) / BN);
  prm.num_tiles = prm.tiles_m * prm.tiles_n * prm.batch;
  prm.k_blocks = static_cast<int>((p.K + BK - 1) / BK);
  prm.alpha = static_cast<float>(p.alpha);
  prm.beta = static_cast<float>(p.beta);
  prm.C_in = p.C;
  prm.ldc = p.ldc;
  prm.strideC = p.strideC;
  prm.bias = p.bias;
  prm.epi = p.epi;
  if (npeers < 0 || npeers > 7) return CUOPX_INVALID_ARGUMENT;
  prm.npeers = npeers;
  for (int i = 0; i < 7; ++i) prm.peer_C[i] = i < npeers ? peers[i] : nullptr;
  // Prefetch reach: the tiles after the first wave, as long as all the first
  // wave warms stays within kPrefetchBudget of L2.
  {
    constexpr int64_t kPrefetchBudget = int64_t(24) << 20;
    prm.wave = device_sm_count() * CPS;
    const int64_t tile_bytes = static_cast<int64_t>(L::A_STAGE + L::B_STAGE) * std::min(prm.k_blocks, STAGES);
    const int64_t reach = (prm.num_tiles + prm.wave - 1) / prm.wave;
    const int64_t cap = std::max<int64_t>(1, kPrefetchBudget / (tile_bytes * prm.wave));
    prm.prefetch_tiles = static_cast<int>(std::max<int64_t>(1, std::min(reach, cap)));
  }

  auto kern = gemm_tc_kernel<T, BN, STAGES, A_MN, B_MN, PEERS, CPS>;
  static std::atomic<bool> attr_set[64] = {};  // per instantiation and device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUOPX_CUDA_ERROR;
  if (!attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess)
      return CUOPX_CUDA_ERROR;
    attr_set[dev].store(true, std::memory_order_relaxed);
  }
  // One CTA per tile; running CTAs take over unlaunched ones' tiles.  The
  // launch may overlap the previous kernel's tail (programmatic dependent
  // launch; the kernel waits before touching global memory).
  const cudaError_t lerr =
      launch_pdl(kern, dim3(static_cast<unsigned>(prm.num_tiles)), dim3(NUM_THREADS), L::ALLOC, stream, mA, mB, mC, prm);
  if (lerr != cudaSuccess) {
    cudaGetLastError();
    return cuda_failure(lerr);
  }
  note_launch(name);
  return check_launch();
}

template <typename T, int BN, int STAGES, int CPS = 1>
int launch_tc_layout(const GemmProblem& p, cudaStream_t stream, const char* name) {
  const bool a_mn = p.transA, b_mn = !p.transB;
  if (!a_mn && b_mn) return launch_tc<T, BN, STAGES, false, true, false, CPS>(p, stream, name);
  if (!a_mn && !b_mn) return launch_tc<T, BN, STAGES, false, false, false, CPS>(p, stream, name);
  if (a_mn && b_mn) return launch_tc<T, BN, STAGES, true, true, false, CPS>(p, stream, name);
  return launch_tc<T, BN, STAGES, true, false, false, CPS>(p, stream, name);
}

}  // namespace

bool gemm_tc_supported(const GemmProblem& p) {
  if (p.dtype != CUOPX_F16 && p.dtype != CUOPX_BF16) return false;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.batch <= 0) return false;
  if (p.M > INT32_MAX || p.N > INT32_MAX || p.K > INT32_MAX || p.batch > 65535) return false;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
  if (!al16(p.A) || !al16(p.B) || !al16(p.C)) return false;
  if (p.lda % 8 || p.ldb % 8 || p.ldc % 8) return false;
  if (p.batch > 1 && (p.strideA % 8 || p.strideB % 8 || p.strideC % 8)) return false;
  if (p.batch > 1 && (p.strideA == 0 || p.strideC == 0)) return false;
  if (p.batch > 1 && p.strideB == 0) return false;  // shared B: generic path
  const int64_t tiles = ((p.M + BM - 1) / BM) * ((p.N + 127) / 128) * p.batch;
  return tiles < (int64_t(1) << 30);
}

int gemm_tc(const GemmProblem& p, cudaStream_t stream, int bn) {
  if (bn == 0 && gemm_tc2_wanted(p)) return gemm_tc2(p, stream);
  if (bn == kTc128x128TwoPerSm) {  // 128 x 128 tiles, two CTAs per SM (2 stages, 256 TMEM columns each)
    return p.dtype == CUOPX_BF16 ? launch_tc_layout<__nv_bfloat16, 128, 2, 2>(p, stream, "gemm_tc_128x128_2cta")
                                 : launch_tc_layout<__half, 128, 2, 2>(p, stream, "gemm_tc_128x128_2cta");
  }
  if (bn == kTc128x64TwoPerSm) {  // 128 x 64 tiles, two CTAs per SM (3 stages, 256 TMEM columns each)
    return p.dtype == CUOPX_BF16 ? launch_tc_layout<__nv_bfloat16, 64, 3, 2>(p, stream, "gemm_tc_128x64_2cta")
                                 : launch_tc_layout<__half, 64, 3, 2>(p, stream, "gemm_tc_128x64_2cta");
  }
  // BN=256 when N fills it and there are at least half as many 128 x 256
  // tiles as SMs (measured on B200: fewer, wider tiles beat a second wave of
  // 128 x 128 tiles); else BN=128.
  const int sms = device_sm_count();
  const int64_t tiles256 = ((p.M + BM - 1) / BM) * ((p.N + 255) / 256) * p.batch;
  const bool wide = bn ? bn == 256 : (p.N > 128 && tiles256 >= sms / 2);
  // Short K loops (one or two 64-deep K blocks per tile, e.g. batched
  // 128 x 128 x 64 heads) are bound by memory and per-tile latency, not by
  // the tensor pipe: two CTAs per SM with two stages each keep as many
  // loads in flight as one CTA with six, and let the next launch's CTAs
  // become resident (and prefetch) while this one drains.  Measured on B200
  // for 4096 x 128x128x64 bf16: 39.6 us vs 43.0 us; 512 batches: 6.7 vs 7.6 us.
  if (bn == 0 && !wide && p.K <= 2 * BK) return gemm_tc(p, stream, kTc128x128TwoPerSm);
  if (p.dtype == CUOPX_BF16) {
    return wide ? launch_tc_layout<__nv_bfloat16, 256, 4>(p, stream, "gemm_tc_128x256")
                : launch_tc_layout<__nv_bfloat16, 128, 6>(p, stream, "gemm_tc_128x128");
  }
  return wide ? launch_tc_layout<__half, 256, 4>(p, stream, "gemm_tc_128x256")
              : launch_tc_layout<__half, 128, 6>(p, stream, "gemm_tc_128x128");
}

// Peer stores are compiled only into the row-major layout of the column-
// sharded linear layer (A K-major, W [K][N] MN-major); other layouts take the
// 2-SM kernel's peer path.
int gemm_tc_peers(const GemmProblem& p, void* const* peers, int npeers, cudaStream_t stream, int bn) {
  if (p.transA || p.transB) return gemm_tc2_peers(p, peers, npeers, stream);
  const bool wide = bn == 256;
  const char* name = wide ? "gemm_tc_128x256_peer" : "gemm_tc_128x128_peer";
  if (p.dtype == CUOPX_BF16) {
    return wide ? launch_tc<__nv_bfloat16, 256, 4, false, true, true>(p, stream, name, peers, npeers)
                : launch_tc<__nv_bfloat16, 128, 6, false, true, true>(p, stream, name, peers, npeers);
  }
  return wide ? launch_tc<__half, 256, 4, false, true, true>(p, stream, name, peers, npeers)
              : launch_tc<__half, 128, 6, false, true, true>(p, stream, name, peers, npeers);
}

}  // namespace cuopx
