// fp32 GEMM on the tensor cores with 3xTF32 (tcgen05.mma kind::tf32).
//
// Each fp32 operand x is split into hi and lo = x - hi (exact in fp32, read
// by the MMA as tf32), and the product is accumulated in fp32 TMEM as
// hi*hi + hi*lo + lo*hi.  An operand in shared memory is its own hi: the
// tensor cores read a 32-bit kind::tf32 operand without its 13 low mantissa
// bits, so the converters write only lo = x - trunc19(x) next to it (one
// store of the tile instead of two); A split into TMEM takes hi = tf32(x)
// rounded to nearest.  The dropped lo*lo term and the tf32 truncation of lo
// bound the per-product error near 2^-20 relative, far inside the fp32
// path's ||C-R||_F/||R||_F <= 1e-5*sqrt(K) (the tests hold it to a tenth of
// that); there is no silent single-pass TF32.  Summation order differs from the
// reference's FFMA chain (gemm.cu:14-42), so results match within that
// tolerance, not bit for bit (the FFMA kernels in gemm_simt.cu are exact).
//
// One persistent CTA per SM, 6 + 4 * CG warps (CG = 2 converter groups):
//   warp 0      TMA producer: fp32 A (128 x 32) and B (BN x 32) tiles into the
//               "hi" buffers of a STAGES-deep ring: 128-byte swizzle for
//               K-major operands, 128-byte swizzle with 32-byte atoms for
//               MN-major ones (the only MN-major layout tf32 MMAs accept).
//   warps 6..   converters, CG groups of 4 taking K blocks in turn: wait
//               for a landed stage; split K-major A straight into TMEM
//               (tcgen05.st, one tile row per thread, the MMAs read A from
//               TMEM), write B's (and an MN-major A's) lo next to the staged
//               tile (same swizzled layout: the split is elementwise);
//               fence, signal the MMA warp.
//   warp 1      TMEM allocator + MMA issuer: 3 x (BK/8) MMAs (M=128, N=BN,
//               K=8) per stage, commit frees the stage / hands off the tile.
//   warps 2..5  epilogue: tcgen05.ld, alpha/beta, swizzled staging, TMA store.
// No TMA multicast.
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int X3_BM = 128;
constexpr int X3_BK = 32;  // 32 fp32 = 128 bytes = one swizzle row
constexpr int X3_EPI_WARPS = 4;
// Converter groups (template parameter CG): group g splits the K blocks
// whose sequence number is g modulo CG, so consecutive stages are split
// concurrently (the split of one stage ends in a TMEM-store wait, which one
// group alone would serialise).  A group is four warps, one per TMEM lane
// quarter, because a warp can only store to its own quarter.  Measured on
// B200: two groups are enough (four gave the same time at 512^3 to 4096^3,
// ~0.7 us per K block at 1024^3 either way).
constexpr int X3_CONV_PER_GROUP = 4;
// Threads per CTA: producer, MMA issuer, 4 epilogue warps, CG converter groups.
__host__ __device__ constexpr int x3_threads(int cg) { return (6 + X3_CONV_PER_GROUP * cg) * 32; }
constexpr int X3_CHUNK = 32;  // epilogue columns per TMA store (32 fp32 = 128 bytes)

struct X3Params {
  int M, N, K, batch;
  int tiles_m, tiles_n, num_tiles, k_blocks;
  float alpha, beta;
  const float* C_in;
  float* C_out;  // the same matrix as C_in (written by plain stores in the pair kernel)
  int64_t ldc, strideC;
  const void* bias;  // CUOPX_EPI_BIAS: N elements of the output type
  int epi;           // CUOPX_EPI_* flags
};

// A_LO: the stage also holds A's lo part in shared memory (MN-major A);
// K-major A is split into TMEM instead, and its stages are 16 KB smaller.
// KSPLIT > 1: a receive area for the other ranks' partial sums of this
// CTA's output columns (split-K over a cluster, see the epilogue).  A
// split-K CTA computes exactly one tile, so its epilogue starts only after
// the last MMA has completed and no load is in flight: the output staging
// and the outgoing partial sums then reuse the stage ring, which leaves room
// for one more stage.
template <int BN, int STAGES, bool A_LO = true, int KSPLIT = 1>
struct X3Smem {
  static constexpr int A_BYTES = X3_BM * X3_BK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * X3_BK * 4;
  static constexpr int STAGE = (A_LO ? 2 : 1) * A_BYTES + 2 * B_BYTES;  // A_hi[, A_lo], B_hi, B_lo
  static constexpr int C_STAGE = 32 * X3_CHUNK * 4;                      // 4 KB
  static constexpr bool C_IN_RING = KSPLIT > 1;
  static_assert(!C_IN_RING || X3_EPI_WARPS * 2 * C_STAGE <= STAGES * STAGE, "staging must fit in the ring");
  static constexpr int OFF_C = C_IN_RING ? 0 : STAGES * STAGE;
  static constexpr int OFF_RECV = C_IN_RING ? STAGES * STAGE : OFF_C + X3_EPI_WARPS * 2 * C_STAGE;
  static constexpr int RECV_SLOT = X3_BM * (BN / KSPLIT) * 4;  // one sender's partial sums
  static constexpr int OFF_SEND = X3_EPI_WARPS * 2 * C_STAGE;   // in the ring, after the staging
  static_assert(!C_IN_RING || OFF_SEND + RECV_SLOT <= STAGES * STAGE, "outgoing sums must fit in the ring");
  static constexpr int OFF_BAR = OFF_RECV + (KSPLIT - 1) * RECV_SLOT;
  // full[S], conv[S], empty[S], acc_full[2], acc_empty[2], drain, recv
  static constexpr int NUM_BARS = 3 * STAGES + 6;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int ALLOC = OFF_MISC + 16 + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget exceeded");
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256, "TMEM allocation must be a power of two >= 32");
  static constexpr int A_OFF = (A_LO ? 2 : 1) * A_BYTES;  // start of B_hi within a stage
  __device__ static unsigned char* a_hi(unsigned char* s, int st) { return s + st * STAGE; }
  __device__ static unsigned char* a_lo(unsigned char* s, int st) { return s + st * STAGE + A_BYTES; }
  __device__ static unsigned char* b_hi(unsigned char* s, int st) { return s + st * STAGE + A_OFF; }
  __device__ static unsigned char* b_lo(unsigned char* s, int st) { return s + st * STAGE + A_OFF + B_BYTES; }
};

__device__ __forceinline__ void x3_tile_coords(int t, const X3Params& p, int& b, int& mt, int& nt) {
  constexpr int G = 8;
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;
  const int r = t - b * per_batch;
  const int span = G * p.tiles_n;
  const int g = r / span;
  const int first_m = g * G;
  const int gsize = min(G, p.tiles_m - first_m);
  const int rr = r - g * span;
  mt = first_m + rr % gsize;
  nt = rr / gsize;
}

__device__ __forceinline__ uint32_t to_tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// x - trunc19(x): the part of x below the tf32 view the tensor cores take
// of it (exact in fp32: both share x's exponent).
__device__ __forceinline__ float tf32_residual(float x) {
  return __fsub_rn(x, __uint_as_float(__float_as_uint(x) & 0xffffe000u));
}

// lo parts of BYTES bytes of staged fp32 at `x` into `lo` by NT threads (the
// staged tile itself is the hi part); the trip count is a compile-time
// constant so every load is issued up front.
template <int BYTES, int NT>
__device__ __forceinline__ void split_tf32_lo(const unsigned char* x, unsigned char* lo, int tid) {
  static_assert(BYTES % (NT * 16) == 0, "split must divide evenly");
  constexpr int ITERS = BYTES / (NT * 16);
  float4 v[ITERS];
#pragma unroll
  for (int i = 0; i < ITERS; ++i) v[i] = *reinterpret_cast<const float4*>(x + (i * NT + tid) * 16);
#pragma unroll
  for (int i = 0; i < ITERS; ++i)
    *reinterpret_cast<float4*>(lo + (i * NT + tid) * 16) =
        make_float4(tf32_residual(v[i].x), tf32_residual(v[i].y), tf32_residual(v[i].z), tf32_residual(v[i].w));
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int CG, int KSPLIT>
__global__ void __launch_bounds__(x3_threads(CG), 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const X3Params p) {
  using L = X3Smem<BN, STAGES, A_MN, KSPLIT>;
  static_assert(KSPLIT == 1 || (BN % (KSPLIT * X3_CHUNK) == 0), "split-K owners take whole store chunks");
  constexpr uint32_t STAGE_TX = static_cast<uint32_t>(L::A_BYTES + L::B_BYTES);
  constexpr uint32_t IDESC = make_idesc(2u /*tf32*/, A_MN, B_MN, X3_BM, BN);
  constexpr uint32_t CHUNK_BYTES = 32 * X3_BK * 4;  // one 32 x 32 fp32 box = 4 KB
  // K-major A is split straight into TMEM (the MMAs read A from there), so
  // only B's split goes back through shared memory.  TMEM: two accumulators
  // (2 x BN columns), then per stage 32 hi + 32 lo columns of A.
  constexpr bool A_TMEM = !A_MN;
  constexpr uint32_t A_COL0 = 2 * BN;
  constexpr uint32_t TMEM_COLS = A_TMEM ? 512u : L::TMEM_COLS;
  static_assert(!A_TMEM || A_COL0 + STAGES * 2 * X3_BK <= 512, "TMEM budget");

  extern __shared__ __align__(1024) unsigned char x3_smem_raw[];
  unsigned char* smem = align_smem_1024(x3_smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* conv = bars + STAGES;
  uint64_t* empty = bars + 2 * STAGES;
  uint64_t* acc_full = bars + 3 * STAGES;
  uint64_t* acc_empty = bars + 3 * STAGES + 2;
  uint64_t* drain = bars + 3 * STAGES + 4;
  uint64_t* recv = bars + 3 * STAGES + 5;  // split K: the other ranks' partial sums have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Work units: tiles, walked persistently (KSPLIT == 1); with KSPLIT > 1
  // one tile per cluster, rank krank of which sums K blocks [kb0, kb1).
  const int krank = KSPLIT > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int unit0 = static_cast<int>(blockIdx.x) / KSPLIT;
  const int ustep = static_cast<int>(gridDim.x) / KSPLIT;
  const int kb0 = krank * p.k_blocks / KSPLIT, kb1 = (krank + 1) * p.k_blocks / KSPLIT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], X3_CONV_PER_GROUP);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], X3_EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(recv, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    // The other ranks' bulk copies complete this many bytes on `recv`.
    if (KSPLIT > 1) mbar_arrive_expect_tx(recv, static_cast<uint32_t>((KSPLIT - 1) * L::RECV_SLOT));
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // Split K: the barriers of every CTA of the cluster are initialised before
  // any rank copies into another (the wait is taken just before that copy;
  // the inits were released by fence.mbarrier_init).
  if constexpr (KSPLIT > 1) cluster_arrive_relaxed();
  const uint32_t tmem_base = *tmem_slot;
  // Global memory only after the previous kernel on the stream has completed
  // (programmatic dependent launch).
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
      for (int t = unit0; t < p.num_tiles && ok; t += ustep) {
        int b, mt, nt;
        x3_tile_coords(t, p, b, mt, nt);
        const int m0 = mt * X3_BM, n0 = nt * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          unsigned char* sa = L::a_hi(smem, stage);
          unsigned char* sb = L::b_hi(smem, stage);
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          const int k0 = kb * X3_BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < X3_BM / 32; ++j)
              tma_load_3d(sa + j * CHUNK_BYTES, &tmA, &full[stage], m0 + 32 * j, k0, b);
          } else {
            tma_load_3d(sa, &tmA, &full[stage], k0, m0, b);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j)
              tma_load_3d(sb + j * CHUNK_BYTES, &tmB, &full[stage], n0 + 32 * j, k0, b);
          } else {
            tma_load_3d(sb, &tmB, &full[stage], k0, n0, b);
          }
          issued_mask |= 1u << stage;
          phase_mask = (phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
      }
      if (ok) grid_launch_dependents();  // all loads issued: the next kernel may start its prologue
      if (!ok) {
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
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------ converters
    constexpr int W = X3_CONV_PER_GROUP;
    constexpr int CPW = X3_BK * 4 / W;  // A columns per warp (TMEM split): 32 or 16
    const int cw = warp - 6;
    const int grp = cw / W;
    const int gtid = threadIdx.x - (6 + grp * W) * 32;  // thread index within the group
    int stage = 0;
    uint32_t phase = 0;
    int seq = 0;
    bool ok = true;
    for (int t = unit0; t < p.num_tiles && ok; t += ustep) {
      for (int kb = kb0; kb < kb1; ++kb, ++seq) {
        if (seq % CG == grp) {
          if (!mbar_wait_bounded(&full[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (A_TMEM) {
            // This warp owns TMEM lane quarter q (tile rows 32q..32q+31) and
            // K columns CPW*h..CPW*h+CPW-1 of the stage; each thread splits
            // its row.
            const int q = warp & 3;
            const int h = (cw % W) >> 2;
            const int r = 32 * q + lane;
            const unsigned char* arow = L::a_hi(smem, stage) + r * 128;  // 128-byte swizzled row
            uint32_t hi[CPW / 16][16], lo[CPW / 16][16];
#pragma unroll
            for (int c = 0; c < CPW / 4; ++c) {
              const float4 v = *reinterpret_cast<const float4*>(arow + ((((CPW / 4) * h + c) ^ (r & 7)) << 4));
              const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int j = 4 * c + i;
                hi[j / 16][j % 16] = to_tf32_rna(e[i]);
                lo[j / 16][j % 16] = __float_as_uint(__fsub_rn(e[i], __uint_as_float(hi[j / 16][j % 16])));
              }
            }
            const uint32_t tcol = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + A_COL0 +
                                  static_cast<uint32_t>(stage * 2 * X3_BK + CPW * h);
#pragma unroll
            for (int u = 0; u < CPW / 16; ++u) {
              tmem_st_32x32b_x16(tcol + 16 * u, hi[u]);
              tmem_st_32x32b_x16(tcol + X3_BK + 16 * u, lo[u]);
            }
            split_tf32_lo<L::B_BYTES, W * 32>(L::b_hi(smem, stage), L::b_lo(smem, stage), gtid);
            tmem_wait_st();
            tc_fence_before_sync();
          } else {
            split_tf32_lo<L::A_BYTES, W * 32>(L::a_hi(smem, stage), L::a_lo(smem, stage), gtid);
            split_tf32_lo<L::B_BYTES, W * 32>(L::b_hi(smem, stage), L::b_lo(smem, stage), gtid);
          }
          fence_proxy_async_shared();  // generic-proxy writes -> visible to the tensor cores
          __syncwarp();
          if (lane == 0) mbar_arrive(&conv[stage]);
        }
        if (++stage == STAGES) stage = 0, phase ^= 1u;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int t = unit0; t < p.num_tiles && ok; t += ustep) {
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, kDevErrWaitTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ready = false;  // this stage's conv phase was seen complete by the early test
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ready && !mbar_wait_bounded(&conv[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const int next = stage + 1 == STAGES ? 0 : stage + 1;
          const uint32_t next_phase = next == 0 ? phase ^ 1u : phase;
          ready = false;
          const uint32_t ah = smem_u32(L::a_hi(smem, stage)), al = smem_u32(L::a_lo(smem, stage));
          const uint32_t bh = smem_u32(L::b_hi(smem, stage)), bl = smem_u32(L::b_lo(smem, stage));
#pragma unroll
          for (int kk = 0; kk < X3_BK / 8; ++kk) {
            // Test the next stage while this one's last MMAs are issued.
            if (kk == X3_BK / 8 - 1 && kb + 1 < kb1) ready = mbar_test_wait(smem_u32(&conv[next]), next_phase);
            // K=8 per MMA: K-major advances 32 bytes in the swizzled row;
            // MN-major advances one 8-row group = 1024 bytes.
            const uint32_t ao = A_MN ? kk * 1024 : kk * 32, bo = B_MN ? kk * 1024 : kk * 32;
            // MN-major tf32 operands use the 32-byte-atom swizzle: 4-row
            // (512-byte) atoms, 32-element chunks CHUNK_BYTES apart.
            const uint64_t dah = A_MN ? make_smem_desc_sw128_32b(ah + ao, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(ah + ao, 16, 1024);
            const uint64_t dal = A_MN ? make_smem_desc_sw128_32b(al + ao, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(al + ao, 16, 1024);
            const uint64_t dbh = B_MN ? make_smem_desc_sw128_32b(bh + bo, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(bh + bo, 16, 1024);
            const uint64_t dbl = B_MN ? make_smem_desc_sw128_32b(bl + bo, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(bl + bo, 16, 1024);
            if constexpr (A_TMEM) {
              const uint32_t ta = tmem_base + A_COL0 + static_cast<uint32_t>(stage * 2 * X3_BK + kk * 8);
              umma_tf32_a_tmem(d_tmem, ta + X3_BK, dbh, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);  // lo*hi first
              umma_tf32_a_tmem(d_tmem, ta, dbl, IDESC, 1u);
              umma_tf32_a_tmem(d_tmem, ta, dbh, IDESC, 1u);
            } else {
              umma_tf32(d_tmem, dal, dbh, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);  // small terms first
              umma_tf32(d_tmem, dah, dbl, IDESC, 1u);
              umma_tf32(d_tmem, dah, dbh, IDESC, 1u);
            }
          }
          issued = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
      if (!ok && issued) {
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
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;
    const int row_in_tile = 32 * q + lane;
    unsigned char* const stage_base = smem + L::OFF_C + (warp - 2) * 2 * L::C_STAGE;  // two buffers
    int sbuf = 0;
    // alpha/beta, bias, ReLU on the fp32 sums of output chunk `ch` of a tile
    // (this thread's row), swizzled staging, TMA store.
    auto finish_chunk = [&](float (&v)[32], int b, int m0, int n0, int ch) {
      const int64_t grow = static_cast<int64_t>(m0) + row_in_tile;
      const int64_t gcol0 = static_cast<int64_t>(n0) + ch * X3_CHUNK;
      if (p.beta != 0.f && grow < p.M) {
        const float* crow = p.C_in + static_cast<int64_t>(b) * p.strideC + grow * p.ldc;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          v[i] = gcol0 + i < p.N ? epi_axpby(p.alpha, v[i], p.beta, crow[gcol0 + i]) : epi_scale(p.alpha, v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = epi_scale(p.alpha, v[i]);
      }
      if (p.epi) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (gcol0 + i < p.N) v[i] = apply_epilogue<float>(v[i], p.bias, gcol0 + i, p.epi);
      }
      if (lane == 0) bulk_wait_group_read<1>();
      __syncwarp();
      unsigned char* sbase = stage_base + sbuf * L::C_STAGE;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(sbase + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tmC, sbase, n0 + ch * X3_CHUNK, m0 + 32 * q, b);
        bulk_commit_group();
      }
      sbuf ^= 1;
    };
    if constexpr (KSPLIT == 1) {
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = unit0; t < p.num_tiles; t += ustep) {
        int b, mt, nt;
        x3_tile_coords(t, p, b, mt, nt);
        if (!mbar_wait_bounded(&acc_full[acc], acc_phase, kDevErrWaitTimeoutAccFull, abort_flag)) break;
        tc_fence_after_sync();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
        for (int ch = 0; ch < BN / X3_CHUNK; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + ch * X3_CHUNK, r);
          tmem_wait_ld();
          if (ch == BN / X3_CHUNK - 1) {
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
          }
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
          finish_chunk(v, b, mt * X3_BM, nt * BN, ch);
        }
        if (++acc == 2) acc = 0, acc_phase ^= 1u;
      }
    } else {
      // Split K: rank r of the cluster owns output columns [r*OWN, (r+1)*OWN)
      // of the tile.  Each warp stages the raw fp32 partial sums of its 32
      // rows in the other rank's columns in the (now idle) stage ring, in
      // the receive layout, and one bulk copy moves them into that rank's
      // receive area (completing on its `recv` barrier).  Once the other
      // rank's sums of this rank's columns have landed, p0 + p1 is formed in
      // rank order 0, 1 — a fixed order, so the result does not depend on
      // timing — and finished.
      static_assert(KSPLIT == 2, "the in-place sum below is the fixed order only for two ranks");
      constexpr int OWN = BN / KSPLIT;
      constexpr int CPO = OWN / X3_CHUNK;  // store chunks per owner
      constexpr uint32_t ROWS_BYTES = 32u * OWN * 4u;  // one warp's rows of a receive slot
      int b = 0, mt = 0, nt = 0;
      x3_tile_coords(unit0, p, b, mt, nt);
      const bool got = unit0 < p.num_tiles &&
                       mbar_wait_bounded(&acc_full[0], 0, kDevErrWaitTimeoutAccFull, abort_flag);
      if (got) tc_fence_after_sync();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
      // Receive rows are OWN fp32 (OWN / 4 16-byte granules); granule g of
      // row r lives at g ^ (r & 15), so a warp's 32 rows spread over banks.
      const uint32_t rsw = static_cast<uint32_t>(row_in_tile & 15);
      const int dst = krank ^ 1;
      unsigned char* send_rows = smem + L::OFF_SEND + 32 * q * OWN * 4;
      unsigned char* send_row = smem + L::OFF_SEND + row_in_tile * OWN * 4;
#pragma unroll 1
      for (int c = 0; c < CPO; ++c) {
        uint32_t r[32];
        if (got) {
          tmem_ld_32x32b_x32(t_row + (dst * CPO + c) * X3_CHUNK, r);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;  // unblocks the other rank; the error is already recorded
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t g = static_cast<uint32_t>(c * 8 + j) ^ rsw;
          *reinterpret_cast<uint4*>(send_row + (g << 4)) = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
        }
      }
      fence_proxy_async_shared();  // staged sums -> visible to the bulk copy
      cluster_wait();              // the other rank's barriers are initialised
      __syncwarp();
      if (lane == 0)
        bulk_copy_to_cluster(map_to_rank(smem + L::OFF_RECV + 32 * q * OWN * 4, static_cast<uint32_t>(dst)),
                             send_rows, ROWS_BYTES, map_to_rank(recv, static_cast<uint32_t>(dst)));
      // This rank's own columns, while the copies are in flight.
      uint32_t own[CPO][32];
      if (got) {
#pragma unroll
        for (int c = 0; c < CPO; ++c) tmem_ld_32x32b_x32(t_row + (krank * CPO + c) * X3_CHUNK, own[c]);
        tmem_wait_ld();
      }
      const bool landed = mbar_wait_bounded(recv, 0, kDevErrWaitTimeoutFull, abort_flag);
      if (got && landed) {
        const unsigned char* rrow = smem + L::OFF_RECV + row_in_tile * OWN * 4;
#pragma unroll
        for (int c = 0; c < CPO; ++c) {
          // Two ranks: the fixed-order sum p0 + p1 is one IEEE addition,
          // which is commutative, so each rank adds the other's part to its
          // own in place.
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(own[c][i]);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 f = *reinterpret_cast<const float4*>(rrow + ((static_cast<uint32_t>(c * 8 + j) ^ rsw) << 4));
            v[4 * j] = __fadd_rn(v[4 * j], f.x);
            v[4 * j + 1] = __fadd_rn(v[4 * j + 1], f.y);
            v[4 * j + 2] = __fadd_rn(v[4 * j + 2], f.z);
            v[4 * j + 3] = __fadd_rn(v[4 * j + 3], f.w);
          }
          finish_chunk(v, b, mt * X3_BM, nt * BN, krank * CPO + c);
        }
      }
    }
    // The bulk stores must have read the staging before the CTA exits; the
    // global writes complete on their own and are visible once the grid has
    // completed (what the next kernel's dependent-launch wait waits for).
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
  }
  // Split K: the other roles complete the early cluster barrier too (the
  // epilogue warps waited on it above).  Then one more: a rank exits only
  // after every copy it sent has landed (the receiver waited for it) and
  // every copy into it has completed.
  if constexpr (KSPLIT > 1) {
    if (warp < 2 || warp >= 6) cluster_wait();
    cluster_sync_all();
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int CG, int KSPLIT>
int launch_x3(const GemmProblem& p, cudaStream_t stream, const char* name) {
  using L = X3Smem<BN, STAGES, A_MN, KSPLIT>;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap mA, mB, mC;
  bool ok = true;
  constexpr auto kMN = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;  // MN-major tf32 layout
  if (A_MN) ok &= make_map_es(&mA, dt, 4, p.A, p.M, p.K, p.batch, p.lda, p.strideA, 32, X3_BK, kMN);
  else ok &= make_map_es(&mA, dt, 4, p.A, p.K, p.M, p.batch, p.lda, p.strideA, X3_BK, X3_BM);
  if (B_MN) ok &= make_map_es(&mB, dt, 4, p.B, p.N, p.K, p.batch, p.ldb, p.strideB, 32, X3_BK, kMN);
  else ok &= make_map_es(&mB, dt, 4, p.B, p.K, p.N, p.batch, p.ldb, p.strideB, X3_BK, BN);
  ok &= make_map_es(&mC, dt, 4, p.C, p.N, p.M, p.batch, p.ldc, p.strideC, X3_CHUNK, 32);
  if (!ok) return CUOPX_CUDA_ERROR;
  X3Params prm;
  prm.M = static_cast<int>(p.M);
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.tiles_m = static_cast<int>((p.M + X3_BM - 1) / X3_BM);
  prm.tiles_n = static_cast<int>((p.N + BN - 1) / BN);
  prm.num_tiles = prm.tiles_m * prm.tiles_n * prm.batch;
  prm.k_blocks = static_cast<int>((p.K + X3_BK - 1) / X3_BK);
  prm.alpha = static_cast<float>(p.alpha);
  prm.beta = static_cast<float>(p.beta);
  prm.C_in = static_cast<const float*>(p.C);
  prm.C_out = static_cast<float*>(p.C);
  prm.ldc = p.ldc;
  prm.strideC = p.strideC;
  prm.bias = p.bias;
  prm.epi = p.epi;
  auto kern = gemm_tf32x3_kernel<BN, STAGES, A_MN, B_MN, CG, KSPLIT>;
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUOPX_CUDA_ERROR;
  if (!attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess)
      return CUOPX_CUDA_ERROR;
    attr_set[dev].store(true, std::memory_order_relaxed);
  }
  cudaError_t err;
  if constexpr (KSPLIT > 1) {  // one cluster of KSPLIT CTAs per tile
    err = launch_pdl_cluster(kern, dim3(static_cast<unsigned>(prm.num_tiles * KSPLIT)), dim3(x3_threads(CG)), L::ALLOC,
                             stream, KSPLIT, mA, mB, mC, prm);
  } else {  // persistent: at most one CTA per SM
    const int grid = std::min(prm.num_tiles, device_sm_count());
    err = launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(x3_threads(CG)), L::ALLOC, stream, mA, mB, mC, prm);
  }
  if (err != cudaSuccess) {
    cudaGetLastError();
    return cuda_failure(err);
  }
  note_launch(name);
  return check_launch();
}

// Stage counts: K-major A (A split in TMEM, smaller stages) runs deeper
// rings — 6 x 64 or 4 x 64 TMEM columns of A next to the accumulators.
template <int BN, int STAGES_TMEM_A, int STAGES_SMEM_A, int CG = 2, int KSPLIT = 1>
int launch_x3_layout(const GemmProblem& p, cudaStream_t stream, const char* name) {
  const bool a_mn = p.transA, b_mn = !p.transB;
  if (!a_mn && b_mn) return launch_x3<BN, STAGES_TMEM_A, false, true, CG, KSPLIT>(p, stream, name);
  if (!a_mn && !b_mn) return launch_x3<BN, STAGES_TMEM_A, false, false, CG, KSPLIT>(p, stream, name);
  if (a_mn && b_mn) return launch_x3<BN, STAGES_SMEM_A, true, true, CG, KSPLIT>(p, stream, name);
  return launch_x3<BN, STAGES_SMEM_A, true, false, CG, KSPLIT>(p, stream, name);
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2) with K split over two pairs.
//
// A cluster of four CTAs owns one 256 x 128 output tile.  CTAs 2h and 2h+1
// form a pair that sums the K blocks of half h; within the pair CTA r holds
// tile rows [128r, 128r+128) (its A rows, split into its own TMEM) and tile
// columns [64r, 64r+64) of B (staged fp32 plus lo, in its own shared memory).
// The even CTA issues M=256, N=128, K=8 MMAs that read both CTAs' A from
// TMEM and both halves of B, and write each CTA's 128 accumulator rows into
// that CTA's TMEM.  Per SM this halves the B traffic of the one-CTA kernel
// (TMA bytes, the split, and the MMAs' shared-memory reads), which is what
// bounds that kernel's K loop.
//   warp 0      TMA producer (each CTA: its A rows and B half, its own `full`)
//   warp 1      TMEM allocation (cta_group::2); on the even CTA the MMA
//               issuer: waits for both CTAs' converters on its `conv`
//               barrier, commits stage release and tile completion to both
//               CTAs of the pair (tcgen05.commit multicast)
//   warps 2..5  epilogue: as the one-CTA split — CTA r of half h finishes
//               output columns [64h, 64h+64) of its 128 rows, after one bulk
//               copy per warp has brought the other half's partial sums of
//               them (from cluster rank r ^ 2) into its `recv` area; the
//               outputs leave through a swizzled staging buffer as plain
//               coalesced stores
//   warps 6..   converters, one group of four per 32-deep sub-block of a
//               stage: A rows into this CTA's TMEM, B lo next to the staged
//               B half; every converter warp arrives on the even CTA's
//               `conv` barrier
// K-major A only (A in TMEM); B either layout.  No TMA multicast.
constexpr int XP_BN = 128;     // pair tile columns (64 of B per CTA)
// A stage is XP_SUB sub-blocks of 32 K (one 128-byte swizzle row each): the
// MMA thread waits once per 24 MMAs.  A wait whose result the issuing thread
// consumes leaves the tensor pipe idle for part of it (the pipe queues about
// one 64-cycle MMA ahead), so fewer, larger stages lose less.
constexpr int XP_SUB = 2;
constexpr int XP_BK = XP_SUB * X3_BK;  // 64
constexpr int XP_STAGES = 3;   // TMEM: 128 accumulator columns + 3 x 128 of A = 512

struct XPSmem {
  static constexpr int A_SUB = X3_BM * X3_BK * 4;          // 16 KB: one 32-deep sub-block of A
  static constexpr int B_SUB = (XP_BN / 2) * X3_BK * 4;    // 8 KB: this CTA's half of B, one sub-block
  static constexpr int A_BYTES = XP_SUB * A_SUB;
  static constexpr int B_BYTES = XP_SUB * B_SUB;
  static constexpr int STAGE = A_BYTES + 2 * B_BYTES;      // A, B (its own hi), B lo
  static constexpr int C_STAGE = 32 * X3_CHUNK * 4;        // 4 KB
  static constexpr int OWN = XP_BN / 2;                    // columns each K half finishes
  static constexpr int RECV_SLOT = X3_BM * OWN * 4;        // 32 KB
  // The epilogue runs after the last MMA, with no load in flight: its
  // output staging and outgoing partial sums reuse the ring.
  static constexpr int OFF_C = 0;
  static constexpr int OFF_SEND = X3_EPI_WARPS * 2 * C_STAGE;
  static_assert(OFF_SEND + RECV_SLOT <= XP_STAGES * STAGE, "epilogue buffers must fit in the ring");
  static constexpr int OFF_RECV = XP_STAGES * STAGE;
  static constexpr int OFF_BAR = OFF_RECV + RECV_SLOT;
  // full[S], conv[S], empty[S], acc_full, drain, recv
  static constexpr int NUM_BARS = 3 * XP_STAGES + 3;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int ALLOC = OFF_MISC + 16 + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget exceeded");
  // Sub-block j of stage st.
  __device__ static unsigned char* a(unsigned char* s, int st, int j) { return s + st * STAGE + j * A_SUB; }
  __device__ static unsigned char* b_hi(unsigned char* s, int st, int j) {
    return s + st * STAGE + A_BYTES + j * B_SUB;
  }
  __device__ static unsigned char* b_lo(unsigned char* s, int st, int j) {
    return s + st * STAGE + A_BYTES + B_BYTES + j * B_SUB;
  }
};

template <bool B_MN, int CG>
__global__ void __launch_bounds__(x3_threads(CG), 1)
    gemm_tf32x3_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const X3Params p) {
  using L = XPSmem;
  constexpr uint32_t STAGE_TX = static_cast<uint32_t>(L::A_BYTES + L::B_BYTES);
  constexpr uint32_t IDESC = make_idesc(2u /*tf32*/, false, B_MN, 2 * X3_BM, XP_BN);
  constexpr uint32_t CHUNK_BYTES = 32 * X3_BK * 4;  // one 32 x 32 fp32 box = 4 KB
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t A_COL0 = XP_BN;  // accumulator: columns [0, 128)
  static_assert(A_COL0 + XP_STAGES * 2 * XP_BK <= TMEM_COLS, "TMEM budget");
  constexpr int OWN = L::OWN;
  constexpr int CPO = OWN / X3_CHUNK;  // store chunks per K half
  constexpr int W = X3_CONV_PER_GROUP;

  extern __shared__ __align__(1024) unsigned char xp_smem_raw[];
  unsigned char* smem = align_smem_1024(xp_smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* conv = bars + XP_STAGES;   // the even CTA's copy counts both CTAs' converters
  uint64_t* empty = bars + 2 * XP_STAGES;
  uint64_t* acc_full = bars + 3 * XP_STAGES;
  uint64_t* drain = bars + 3 * XP_STAGES + 1;
  uint64_t* recv = bars + 3 * XP_STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0..3
  const int pr = static_cast<int>(rank & 1u);  // row half within the pair; 0 issues the MMAs
  const int kh = static_cast<int>(rank >> 1);  // K half
  const uint32_t even = rank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << even);
  const int tile = static_cast<int>(blockIdx.x) / 4;
  const int kb0 = kh * p.k_blocks / 2, kb1 = (kh + 1) * p.k_blocks / 2;
  int b, mt, nt;
  x3_tile_coords(tile, p, b, mt, nt);
  const int m0 = mt * 2 * X3_BM + pr * X3_BM;  // this CTA's rows
  const int n0 = nt * XP_BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < XP_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 2 * CG * W);  // every converter warp of both CTAs
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    mbar_init(recv, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    mbar_arrive_expect_tx(recv, static_cast<uint32_t>(L::RECV_SLOT));  // the other K half's bulk copies
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  __syncthreads();  // barrier inits visible in the CTA
  // The producer starts loading at once; the pair's TMEM allocation (which
  // the other roles need) runs meanwhile, published to them on named
  // barrier 1.
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    tc_fence_before_sync();
  }
  if (warp != 0) {
    named_bar_sync(1, x3_threads(CG) - 32);
    tc_fence_after_sync();
  }
  // Barrier inits and TMEM allocations are published to the cluster here and
  // waited for just before each role's first cross-CTA operation, so the
  // first loads overlap the cluster barrier.  Only warp 1 (the TMEM
  // allocation) needs a releasing arrival; the barrier inits were released by
  // fence.mbarrier_init.
  if (warp == 1) cluster_arrive();
  else cluster_arrive_relaxed();
  const uint32_t tmem_base = warp != 0 ? *tmem_slot : 0u;
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, phase_mask = 0;
      bool ok = true;
      const int nb = n0 + pr * (XP_BN / 2);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], STAGE_TX);
#pragma unroll
        for (int j = 0; j < XP_SUB; ++j) {
          const int k0 = kb * XP_BK + j * X3_BK;  // past K: the TMA fills zeros
          tma_load_3d(L::a(smem, stage, j), &tmA, &full[stage], k0, m0, b);
          unsigned char* sb = L::b_hi(smem, stage, j);
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < (XP_BN / 2) / 32; ++c)
              tma_load_3d(sb + c * CHUNK_BYTES, &tmB, &full[stage], nb + 32 * c, k0, b);
          } else {
            tma_load_3d(sb, &tmB, &full[stage], k0, nb, b);
          }
        }
        issued_mask |= 1u << stage;
        phase_mask = (phase_mask & ~(1u << stage)) | (phase << stage);
        if (++stage == XP_STAGES) stage = 0, phase ^= 1u;
      }
      if (ok) {
        grid_launch_dependents();  // all loads issued: the next kernel may start its prologue
        // Wait until every stage's last use is released, so no multicast
        // commit is still on its way to this CTA's barriers at exit.
        for (int i = 0; i < XP_STAGES; ++i) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) break;
          if (++stage == XP_STAGES) stage = 0, phase ^= 1u;
        }
      } else {
        for (int s = 0; s < XP_STAGES; ++s) {
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
      }
    }
    cluster_wait();
  } else if (warp >= 6) {
    // ------------------------------------------------------------ converters
    cluster_wait();  // the even CTA's conv barriers are initialised
    const int cw = warp - 6;
    const int grp = cw / W;
    const int gtid = threadIdx.x - (6 + grp * W) * 32;
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int r = 32 * q + lane;
    // Group g splits sub-block g of every stage (A rows into TMEM, B's lo),
    // so a stage is ready after half the split work of one group alone.
    static_assert(CG == XP_SUB, "one converter group per sub-block");
    const int sb = grp;
    int stage = 0;
    uint32_t phase = 0;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait_bounded(&full[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) break;
      // Row r of A sub-block sb (128 swizzled bytes) -> hi, lo into TMEM
      // stage columns [64 sb, 64 sb + 32) (hi) and [64 sb + 32, 64 sb + 64) (lo).
      const unsigned char* arow = L::a(smem, stage, sb) + r * 128;
      uint32_t hi[2][16], lo[2][16];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 v = *reinterpret_cast<const float4*>(arow + ((c ^ (r & 7)) << 4));
        const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = 4 * c + i;
          hi[j / 16][j % 16] = to_tf32_rna(e[i]);
          lo[j / 16][j % 16] = __float_as_uint(__fsub_rn(e[i], __uint_as_float(hi[j / 16][j % 16])));
        }
      }
      const uint32_t tcol = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + A_COL0 +
                            static_cast<uint32_t>(stage * 2 * XP_BK + sb * 2 * X3_BK);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        tmem_st_32x32b_x16(tcol + 16 * u, hi[u]);
        tmem_st_32x32b_x16(tcol + X3_BK + 16 * u, lo[u]);
      }
      split_tf32_lo<L::B_SUB, W * 32>(L::b_hi(smem, stage, sb), L::b_lo(smem, stage, sb), gtid);
      tmem_wait_st();
      tc_fence_before_sync();
      fence_proxy_async_shared();  // generic-proxy writes -> visible to the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(map_to_rank(&conv[stage], even));
      if (++stage == XP_STAGES) stage = 0, phase ^= 1u;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    cluster_wait();  // the odd CTA's TMEM and barriers are ready
    if (pr == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      bool ready = false;  // this stage's conv phase was seen complete by the early test
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!ready && !mbar_wait_cluster_bounded(&conv[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const int next = stage + 1 == XP_STAGES ? 0 : stage + 1;
        const uint32_t next_phase = next == 0 ? phase ^ 1u : phase;
        ready = false;
#pragma unroll
        for (int sb = 0; sb < XP_SUB; ++sb) {
          const uint32_t bh = smem_u32(L::b_hi(smem, stage, sb)), bl = smem_u32(L::b_lo(smem, stage, sb));
#pragma unroll
          for (int kk = 0; kk < X3_BK / 8; ++kk) {
            // Test the next stage while this one's last MMAs are issued.
            if (sb == XP_SUB - 1 && kk == X3_BK / 8 - 1 && kb + 1 < kb1)
              ready = mbar_test_wait_cluster(smem_u32(&conv[next]), next_phase);
            const uint32_t bo = B_MN ? kk * 1024 : kk * 32;
            const uint64_t dbh = B_MN ? make_smem_desc_sw128_32b(bh + bo, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(bh + bo, 16, 1024);
            const uint64_t dbl = B_MN ? make_smem_desc_sw128_32b(bl + bo, CHUNK_BYTES, 512)
                                      : make_smem_desc_sw128(bl + bo, 16, 1024);
            const uint32_t ta =
                tmem_base + A_COL0 + static_cast<uint32_t>(stage * 2 * XP_BK + sb * 2 * X3_BK + kk * 8);
            umma_tf32_pair_a_tmem(tmem_base, ta + X3_BK, dbh, IDESC, (kb > kb0 || sb > 0 || kk > 0) ? 1u : 0u);
            umma_tf32_pair_a_tmem(tmem_base, ta, dbl, IDESC, 1u);  // lo*hi first, then hi*lo, hi*hi
            umma_tf32_pair_a_tmem(tmem_base, ta, dbh, IDESC, 1u);
          }
        }
        issued = true;
        umma_commit_pair_mask(&empty[stage], pair_mask);
        if (++stage == XP_STAGES) stage = 0, phase ^= 1u;
      }
      if (ok) {
        umma_commit_pair_mask(acc_full, pair_mask);
      } else if (issued) {
        umma_commit_pair_mask(drain, static_cast<uint16_t>(1u << rank));
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
    // ------------------------------------------------------------ epilogue (warps 2..5)
    cluster_wait();  // the other K half's recv barrier is initialised
    const int q = warp & 3;
    const int row_in_tile = 32 * q + lane;
    unsigned char* const stage = smem + L::OFF_C + (warp - 2) * L::C_STAGE;  // this warp's 32 x 32 staging
    const bool got = mbar_wait_bounded(acc_full, 0, kDevErrWaitTimeoutAccFull, abort_flag);
    if (got) tc_fence_after_sync();
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    // Receive rows are OWN fp32; granule g of row r lives at g ^ (r & 15).
    const uint32_t rsw = static_cast<uint32_t>(row_in_tile & 15);
    const uint32_t dst = rank ^ 2u;  // same rows, other K half
    unsigned char* send_row = smem + L::OFF_SEND + row_in_tile * OWN * 4;
#pragma unroll 1
    for (int c = 0; c < CPO; ++c) {
      uint32_t v[32];
      if (got) {
        tmem_ld_32x32b_x32(t_row + ((kh ^ 1) * CPO + c) * X3_CHUNK, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;  // unblocks the other half; the error is already recorded
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t g = static_cast<uint32_t>(c * 8 + j) ^ rsw;
        *reinterpret_cast<uint4*>(send_row + (g << 4)) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
    }
    fence_proxy_async_shared();  // staged sums -> visible to the bulk copy
    __syncwarp();
    if (lane == 0)
      bulk_copy_to_cluster(map_to_rank(smem + L::OFF_RECV + 32 * q * OWN * 4, dst),
                           smem + L::OFF_SEND + 32 * q * OWN * 4, 32u * OWN * 4u, map_to_rank(recv, dst));
    const bool landed = mbar_wait_bounded(recv, 0, kDevErrWaitTimeoutFull, abort_flag);
    if (got && landed) {
      const unsigned char* rrow = smem + L::OFF_RECV + row_in_tile * OWN * 4;
      const int64_t grow = static_cast<int64_t>(m0) + row_in_tile;
#pragma unroll
      for (int c = 0; c < CPO; ++c) {
        // Two K halves: p0 + p1 is one IEEE addition (commutative), the
        // same on both sides; the result does not depend on timing.
        uint32_t own[32];
        tmem_ld_32x32b_x32(t_row + (kh * CPO + c) * X3_CHUNK, own);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(own[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 f = *reinterpret_cast<const float4*>(rrow + ((static_cast<uint32_t>(c * 8 + j) ^ rsw) << 4));
          v[4 * j] = __fadd_rn(v[4 * j], f.x);
          v[4 * j + 1] = __fadd_rn(v[4 * j + 1], f.y);
          v[4 * j + 2] = __fadd_rn(v[4 * j + 2], f.z);
          v[4 * j + 3] = __fadd_rn(v[4 * j + 3], f.w);
        }
        const int64_t gcol0 = static_cast<int64_t>(n0) + (kh * CPO + c) * X3_CHUNK;
        if (p.beta != 0.f && grow < p.M) {
          const float* crow = p.C_in + static_cast<int64_t>(b) * p.strideC + grow * p.ldc;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            v[i] = gcol0 + i < p.N ? epi_axpby(p.alpha, v[i], p.beta, crow[gcol0 + i]) : epi_scale(p.alpha, v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = epi_scale(p.alpha, v[i]);
        }
        if (p.epi) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (gcol0 + i < p.N) v[i] = apply_epilogue<float>(v[i], p.bias, gcol0 + i, p.epi);
        }
        // Transpose through shared memory (rows swizzled by 16-byte granule)
        // so that each store instruction writes four whole 128-byte rows:
        // plain stores, with nothing to wait for before the CTA exits.
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        __syncwarp();
        const int c16 = lane & 7;
        const int64_t gcol = gcol0 + 4 * c16;
        float* const cbase = p.C_out + static_cast<int64_t>(b) * p.strideC;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3);
          const int64_t grow_r = static_cast<int64_t>(m0) + 32 * q + r;
          const float4 w = *reinterpret_cast<const float4*>(stage + r * 128 + ((c16 ^ (r & 7)) << 4));
          if (grow_r < p.M && gcol < p.N) {
            float* dst = cbase + grow_r * p.ldc + gcol;
            if (gcol + 3 < p.N) {
              *reinterpret_cast<float4*>(dst) = w;
            } else {
              dst[0] = w.x;
              if (gcol + 1 < p.N) dst[1] = w.y;
              if (gcol + 2 < p.N) dst[2] = w.z;
            }
          }
        }
        __syncwarp();
      }
    }
  }

  // A CTA exits only after every copy it sent has landed (its receiver
  // waited for it), every copy into it has completed, and its pair partner
  // is done with its TMEM.  (Every role has completed the early cluster
  // barrier above.)
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

template <bool B_MN>
int launch_x3_pair(const GemmProblem& p, cudaStream_t stream, const char* name) {
  using L = XPSmem;
  constexpr int CG = 2;
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap mA, mB;
  bool ok = true;
  constexpr auto kMN = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;  // MN-major tf32 layout
  ok &= make_map_es(&mA, dt, 4, p.A, p.K, p.M, p.batch, p.lda, p.strideA, X3_BK, X3_BM);
  if (B_MN) ok &= make_map_es(&mB, dt, 4, p.B, p.N, p.K, p.batch, p.ldb, p.strideB, 32, X3_BK, kMN);
  else ok &= make_map_es(&mB, dt, 4, p.B, p.K, p.N, p.batch, p.ldb, p.strideB, X3_BK, XP_BN / 2);
  if (!ok) return CUOPX_CUDA_ERROR;
  X3Params prm;
  prm.M = static_cast<int>(p.M);
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.tiles_m = static_cast<int>((p.M + 2 * X3_BM - 1) / (2 * X3_BM));
  prm.tiles_n = static_cast<int>((p.N + XP_BN - 1) / XP_BN);
  prm.num_tiles = prm.tiles_m * prm.tiles_n * prm.batch;
  prm.k_blocks = static_cast<int>((p.K + XP_BK - 1) / XP_BK);  // 64-deep stages
  prm.alpha = static_cast<float>(p.alpha);
  prm.beta = static_cast<float>(p.beta);
  prm.C_in = static_cast<const float*>(p.C);
  prm.C_out = static_cast<float*>(p.C);
  prm.ldc = p.ldc;
  prm.strideC = p.strideC;
  prm.bias = p.bias;
  prm.epi = p.epi;
  auto kern = gemm_tf32x3_pair_kernel<B_MN, CG>;
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUOPX_CUDA_ERROR;
  if (!attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess)
      return CUOPX_CUDA_ERROR;
    attr_set[dev].store(true, std::memory_order_relaxed);
  }
  // One cluster of four CTAs per 256 x 128 tile.
  const cudaError_t err = launch_pdl_cluster(kern, dim3(static_cast<unsigned>(prm.num_tiles * 4)), dim3(x3_threads(CG)),
                                             L::ALLOC, stream, 4, mA, mB, prm);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return cuda_failure(err);
  }
  note_launch(name);
  return check_launch();
}

}  // namespace

bool gemm_tf32x3_supported(const GemmProblem& p) {
  if (p.dtype != CUOPX_F32) return false;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.batch <= 0) return false;
  if (p.M > INT32_MAX || p.N > INT32_MAX || p.K > INT32_MAX || p.batch > 65535) return false;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) % 16) == 0; };
  if (!al16(p.A) || !al16(p.B) || !al16(p.C)) return false;
  if (p.lda % 4 || p.ldb % 4 || p.ldc % 4) return false;
  if (p.batch > 1 && (p.strideA % 4 || p.strideB % 4 || p.strideC % 4 || p.strideA == 0 || p.strideB == 0 ||
                      p.strideC == 0))
    return false;
  return true;
}

int gemm_tf32x3(const GemmProblem& p, cudaStream_t stream, int bn) {
  if (bn == 0) {
    const int sms = device_sm_count();
    const int64_t tiles128 = ((p.M + X3_BM - 1) / X3_BM) * ((p.N + 127) / 128) * p.batch;
    const int64_t tiles_pair = ((p.M + 2 * X3_BM - 1) / (2 * X3_BM)) * ((p.N + XP_BN - 1) / XP_BN) * p.batch;
    const int64_t k_blocks = (p.K + X3_BK - 1) / X3_BK;
    // Too few tiles to fill the part but a long K loop: split K in two.
    // With K-major A, 256 x 128 tiles on CTA pairs (clusters of four CTAs),
    // which halve each SM's share of B; otherwise 128 x 128 tiles on
    // clusters of two CTAs.
    if (p.N > 64 && !p.transA && tiles_pair * 4 <= sms && k_blocks >= 8) {
      bn = kTf32x3PairSplitK2;
    } else if (p.N > 64 && tiles128 * 2 <= sms && k_blocks >= 8) {
      bn = kTf32x3SplitK2;
    } else {
      // 128 x 128 tiles halve B traffic per FLOP; measured on B200 they win
      // from about two thirds of an SM wave of them.
      bn = (p.N > 64 && tiles128 * 3 >= sms * 2) ? 128 : 64;
    }
  }
  // Each K half needs at least one K block of its own (64 deep in the pair
  // kernel); the pair kernel takes K-major A only.
  if (bn == kTf32x3PairSplitK2 && (p.transA || (p.K + XP_BK - 1) / XP_BK < 2)) bn = kTf32x3SplitK2;
  if (bn == kTf32x3SplitK2 && (p.K + X3_BK - 1) / X3_BK < 2) bn = 128;
  if (bn == kTf32x3PairSplitK2)
    return p.transB ? launch_x3_pair<false>(p, stream, "gemm_tf32x3_256x128_pair_k2")
                    : launch_x3_pair<true>(p, stream, "gemm_tf32x3_256x128_pair_k2");
  if (bn == kTf32x3SplitK2) return launch_x3_layout<128, 4, 3, 2, 2>(p, stream, "gemm_tf32x3_128x128_k2");
  if (bn == 128) return launch_x3_layout<128, 4, 3>(p, stream, "gemm_tf32x3_128x128");
  return launch_x3_layout<64, 6, 4>(p, stream, "gemm_tf32x3_128x64");
}

}  // namespace cuopx
