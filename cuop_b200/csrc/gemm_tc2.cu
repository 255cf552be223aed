// Two-SM tcgen05 GEMM (cta_group::2) for large fp16/bf16 problems.
//
// A cluster of two CTAs on two SMs owns a 256 x PBN output tile (PBN = 128,
// 256 or 512).  A slot is SLOT = min(PBN, 256) accumulator columns, the N of
// one MMA.  CTA r of the pair loads rows [128r, 128r+128) of the A tile and,
// for each slot h of the tile, columns [SLOT h + SLOT/2 r, SLOT h + SLOT/2 (r+1))
// of the B tile into its own shared memory; one tcgen05.mma.cta_group::2
// (M=256, N=SLOT, K=16) per slot, issued by the even CTA, reads both CTAs'
// halves and writes each CTA's 128 accumulator rows of that slot into the
// CTA's TMEM (512 / SLOT slots).  Per SM this halves the shared-memory
// operand traffic of the 1-SM kernel of the same tile width.
//   PBN = 128: 7-stage ring of 24 KB, four TMEM slots rotating between
//              tiles; a tile's outputs are ready after half the MMA time of
//              a 256 x 256 tile, which the peer-store path can use to start
//              its NVLink traffic earlier.
//   PBN = 256: 6-stage ring of 32 KB; the two TMEM slots alternate between
//              tiles, so the epilogue of a tile overlaps the next one.
//   PBN = 512: 4-stage ring of 48 KB; a tile fills both slots, so each K
//              block pulls 25 % fewer operand bytes from L2 per FLOP and
//              covers twice the MMA time per stage.  The epilogue drains
//              slot 0, releases it, then slot 1; the next tile's MMAs into
//              slot 0 start as soon as slot 0 is free and its first MMAs
//              into slot 1 wait only for the rest of the drain.
//
//   warp 0      TMA producer (both CTAs): loads complete on the LEADER's
//               `full` mbarrier (.cta_group::2); the leader posts the
//               expected byte count for both halves.
//   warp 1      TMEM allocation (cta_group::2, both CTAs); on the leader, the
//               MMA issuer: waits `full`, issues 4 MMAs per slot per stage,
//               commits stage release to `empty` and tile completion to
//               `acc_full` in BOTH CTAs (tcgen05.commit multicast).
//   warps 2..5  epilogue (both CTAs): own TMEM rows -> alpha/beta -> swizzled
//               staging -> TMA store; then arrive on the leader's `acc_empty`.
// Tile scheduling: one cluster per pair tile is launched; the leader asks the
// hardware (clusterlaunchcontrol.try_cancel, answer in its own shared
// memory) to cancel a cluster that has not been launched yet and takes over
// its tile, then forwards the answer into the partner CTA's ring slot with a
// shared::cluster store and a remote release-arrive.  Every role of both
// CTAs walks the same tile sequence; the partner's roles release a slot by
// arriving on the leader's clc_empty barrier.
// No TMA multicast: every CTA loads its own halves.  Cluster barriers bracket
// the kernel so no CTA exits while its peer may still touch its shared memory.
#include "common.cuh"
#include "dispatch.h"

namespace cuopx {

namespace {

constexpr int P_BM = 128;  // rows per CTA (pair: 256)
constexpr int P_BK = 64;
constexpr int P_THREADS = 192;
constexpr int P_EPI_WARPS = 4;
constexpr int P_CHUNK = 64;
constexpr uint32_t P_TMEM_COLS = 512;
constexpr int P_MAX_SLOTS = 4;    // TMEM slots at the narrowest tile (128 columns each)
constexpr int P_GROUP_M = 8;      // pair-row tiles per raster group
// Scheduler ring depth (> the producers' lead over the epilogue, in tiles).
constexpr int P_CLC_SLOTS = 16;
// Arrivals on the leader's clc_empty per slot: leader producer, MMA issuer and
// epilogue warps, plus the partner's producer and epilogue warps (remote).
constexpr int P_CLC_READERS = (2 + P_EPI_WARPS) + (1 + P_EPI_WARPS);

template <int PBN>
struct PairCfg {
  static_assert(PBN == 128 || PBN == 256 || PBN == 512, "pair tile width");
  static constexpr int SLOT = PBN < 256 ? PBN : 256;               // accumulator columns of one MMA (its N)
  static constexpr int SLOTS = static_cast<int>(P_TMEM_COLS) / SLOT;  // TMEM slots
  static constexpr int SPT = PBN / SLOT;                           // TMEM slots per tile
  static constexpr int STAGES = PBN == 128 ? 7 : (SPT == 1 ? 6 : 4);
};

template <int PBN>
struct PairSmem {
  static constexpr int STAGES = PairCfg<PBN>::STAGES;
  static constexpr int A_STAGE = P_BM * P_BK * 2;               // 16 KB
  static constexpr int B_PIECE = (PairCfg<PBN>::SLOT / 2) * P_BK * 2;  // this CTA's half of one slot
  static constexpr int B_STAGE = PairCfg<PBN>::SPT * B_PIECE;
  static constexpr int C_STAGE = 32 * P_CHUNK * 2;              // 4 KB
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = STAGES * A_STAGE;
  static constexpr int OFF_C = OFF_B + STAGES * B_STAGE;
  static constexpr int OFF_BAR = OFF_C + P_EPI_WARPS * 2 * C_STAGE;
  // full[S], empty[S], acc_full[SLOTS], acc_empty[SLOTS], drain
  static constexpr int NUM_BARS = 2 * STAGES + 2 * PairCfg<PBN>::SLOTS + 1;
  // Tile-scheduler ring: P_CLC_SLOTS 16-byte launch-control responses, then
  // clc_full[P_CLC_SLOTS] and clc_empty[P_CLC_SLOTS] mbarriers.
  static constexpr int OFF_CLC = (OFF_BAR + NUM_BARS * 8 + 15) / 16 * 16;
  static constexpr int OFF_CLC_BAR = OFF_CLC + P_CLC_SLOTS * 16;
  static constexpr int OFF_MISC = OFF_CLC_BAR + 2 * P_CLC_SLOTS * 8;
  static constexpr int ALLOC = OFF_MISC + 16 + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget exceeded");
};

constexpr int P_MAX_PEERS = 7;  // one node: up to 8 ranks

struct PairParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, num_tiles, k_blocks;  // tiles are 256 x PBN pair tiles
  float alpha, beta;
  const void* C_in;
  int64_t ldc, strideC;
  // Peer-store all-gather: each staged output chunk is also written to
  // peer_C[i] (same row stride ldc, same column offset) for i < npeers.
  int npeers;
  void* peer_C[P_MAX_PEERS];
  const void* bias;  // CUOPX_EPI_BIAS: N elements of the output type
  int epi;           // CUOPX_EPI_* flags
};


// Next pair tile from a completed launch-control response (the cancelled
// cluster's first CTA index / 2); false when none was left.
__device__ __forceinline__ bool clc_next_pair_tile(const void* resp, int num_tiles, int& next) {
  int ctaid = 0;
  if (!clc_query(resp, ctaid)) return false;
  next = ctaid >> 1;
  if (ctaid < 0 || next >= num_tiles) {
    record_device_error(kDevErrSchedule);
    return false;
  }
  return true;
}


// TMA load into this CTA's smem, completing bytes on the mbarrier at a
// shared::cluster address (the leader's), no multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const void* tmap, uint32_t mbar_cluster, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(mbar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (same offset) in both CTAs of the pair when all prior
// tcgen05 ops of this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void pair_tile_coords(int t, const PairParams& p, int& b, int& mt, int& nt) {
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;
  const int r = t - b * per_batch;
  const int span = P_GROUP_M * p.tiles_n;
  const int g = r / span;
  const int first_m = g * P_GROUP_M;
  const int gsize = min(P_GROUP_M, p.tiles_m - first_m);
  const int rr = r - g * span;
  mt = first_m + rr % gsize;
  nt = rr / gsize;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2_pair(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2_pair<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2_pair<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <typename T, bool A_MN, bool B_MN, int PBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const PairParams p) {
  using L = PairSmem<PBN>;
  constexpr int SPT = PairCfg<PBN>::SPT;
  constexpr int P_STAGES = PairCfg<PBN>::STAGES;
  constexpr int P_SLOT_COLS = PairCfg<PBN>::SLOT;
  constexpr int P_SLOTS = PairCfg<PBN>::SLOTS;
  constexpr int CHUNKS_PER_SLOT = P_SLOT_COLS / P_CHUNK;
  constexpr uint32_t PAIR_TX = 2u * static_cast<uint32_t>(L::A_STAGE + L::B_STAGE);
  constexpr uint32_t AB_FMT = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t IDESC = make_idesc(AB_FMT, A_MN, B_MN, 2 * P_BM, P_SLOT_COLS);

  extern __shared__ __align__(1024) unsigned char pair_smem_raw[];
  unsigned char* smem = align_smem_1024(pair_smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* full = bars;
  uint64_t* empty = bars + P_STAGES;
  uint64_t* acc_full = bars + 2 * P_STAGES;
  uint64_t* acc_empty = bars + 2 * P_STAGES + P_SLOTS;
  uint64_t* drain = bars + 2 * P_STAGES + 2 * P_SLOTS;
  unsigned char* clc_resp = smem + L::OFF_CLC;
  uint64_t* clc_full = reinterpret_cast<uint64_t*>(smem + L::OFF_CLC_BAR);
  uint64_t* clc_empty = clc_full + P_CLC_SLOTS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);   // leader: its own arrive.expect_tx; both CTAs' bytes
      mbar_init(&empty[s], 1);  // one multicast commit per phase
    }
    for (int a = 0; a < P_SLOTS; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * P_EPI_WARPS);  // leader's copy: 4 local + 4 remote arrivals
    }
    for (int c = 0; c < P_CLC_SLOTS; ++c) {
      mbar_init(&clc_full[c], 1);  // leader: its expect_tx; partner: the leader's forward
      mbar_init(&clc_empty[c], P_CLC_READERS);  // used on the leader only
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(P_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // barrier inits and TMEM allocation visible to the peer
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  // Global memory (and peers' memory) only after the previous kernel on the
  // stream has completed (programmatic dependent launch).
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Abort bookkeeping, one bit per stage: loaded at least once, and the
      // parity of the last phase loaded.
      uint32_t issued_mask = 0, phase_mask = 0;
      bool clc_pending = false;
      int cs = 0;
      uint32_t cpar = 0;
      int t = pair;
      for (int seq = 0; ok; ++seq) {
        cs = seq % P_CLC_SLOTS;
        cpar = static_cast<uint32_t>(seq / P_CLC_SLOTS) & 1u;
        if (leader) {
          // Ask for the pair tile after this one (answer by the end of it).
          if (!mbar_wait_bounded(&clc_empty[cs], cpar ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&clc_full[cs], 16);
          clc_try_cancel(clc_resp + cs * 16, &clc_full[cs]);
          clc_pending = true;
        }
        int b, mt, nt;
        pair_tile_coords(t, p, b, mt, nt);
        const int m0 = mt * 2 * P_BM + static_cast<int>(rank) * P_BM;
        const int n0 = nt * PBN + static_cast<int>(rank) * (P_SLOT_COLS / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], PAIR_TX);
          const uint32_t mbar = map_to_rank(&full[stage], 0);
          unsigned char* sa = smem + L::OFF_A + stage * L::A_STAGE;
          unsigned char* sb = smem + L::OFF_B + stage * L::B_STAGE;
          const int k0 = kb * P_BK;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < P_BM / 64; ++j) tma_load_3d_pair(sa + j * (64 * P_BK * 2), &tmA, mbar, m0 + 64 * j, k0, b);
          } else {
            tma_load_3d_pair(sa, &tmA, mbar, k0, m0, b);
          }
#pragma unroll
          for (int h = 0; h < SPT; ++h) {
            unsigned char* sbh = sb + h * L::B_PIECE;
            const int n0h = n0 + h * P_SLOT_COLS;
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < (P_SLOT_COLS / 2) / 64; ++j)
                tma_load_3d_pair(sbh + j * (64 * P_BK * 2), &tmB, mbar, n0h + 64 * j, k0, b);
            } else {
              tma_load_3d_pair(sbh, &tmB, mbar, k0, n0h, b);
            }
          }
          issued_mask |= 1u << stage;
          phase_mask = (phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == P_STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        int next = 0;
        bool more;
        if (leader) {
          if (!mbar_wait_bounded(&clc_full[cs], cpar, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          clc_pending = false;
          // Forward the answer to the partner's slot, then release it there.
          const uint4 r = *reinterpret_cast<const uint4*>(clc_resp + cs * 16);
          st_cluster_v4(map_to_rank(clc_resp + cs * 16, 1), r);
          mbar_arrive_cluster(map_to_rank(&clc_full[cs], 1));
          more = clc_next_pair_tile(clc_resp + cs * 16, p.num_tiles, next);
          mbar_arrive(&clc_empty[cs]);
        } else {
          if (!mbar_wait_cluster_bounded(&clc_full[cs], cpar, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          more = clc_next_pair_tile(clc_resp + cs * 16, p.num_tiles, next);
          mbar_arrive_cluster(map_to_rank(&clc_empty[cs], 0));
        }
        if (!more) {
          grid_launch_dependents();  // all loads issued: the next kernel may start its prologue
          break;
        }
        t = next;
      }
      if (ok) {
        // Tail: wait until the leader has released every stage, so no
        // multicast commit can still be on its way to this CTA's barriers.
        for (int i = 0; i < P_STAGES; ++i) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, kDevErrWaitTimeoutEmpty, abort_flag)) break;
          if (++stage == P_STAGES) stage = 0, phase ^= 1u;
        }
      } else if (leader) {
        // Abort: let every phase this pair issued land (the leader's barrier
        // counts both CTAs' bytes), and the outstanding launch-control
        // answer, before the cluster exits.
        for (int s = 0; s < P_STAGES; ++s) {
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
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;              // first TMEM slot of the tile (rotates when SPT == 1)
      uint32_t empty_bits = 0;  // bit s: parity of slot s's next acc_empty phase
      bool ok = true, issued = false;
      for (int seq = 0; ok; ++seq) {
        const int s0 = SPT == 1 ? acc : 0;
        if (!mbar_wait_bounded(&acc_empty[s0], ((empty_bits >> s0) & 1u) ^ 1u, kDevErrWaitTimeoutAccEmpty,
                               abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, kDevErrWaitTimeoutFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sa = smem_u32(smem + L::OFF_A + stage * L::A_STAGE);
          const uint32_t sb = smem_u32(smem + L::OFF_B + stage * L::B_STAGE);
#pragma unroll
          for (int h = 0; h < SPT; ++h) {
            const int slot = s0 + h;
            if (h > 0 && kb == 0) {
              // The rest of the previous tile's drain: the epilogue releases
              // slot h after slot 0.
              if (!mbar_wait_bounded(&acc_empty[slot], ((empty_bits >> slot) & 1u) ^ 1u, kDevErrWaitTimeoutAccEmpty,
                                     abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after_sync();
            }
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * P_SLOT_COLS);
            const uint32_t sbh = sb + static_cast<uint32_t>(h * L::B_PIECE);
#pragma unroll
            for (int kk = 0; kk < P_BK / 16; ++kk) {
              const uint64_t ad = A_MN ? make_smem_desc_sw128(sa + kk * 2048, 64 * P_BK * 2, 1024)
                                       : make_smem_desc_sw128(sa + kk * 32, 16, 1024);
              const uint64_t bd = B_MN ? make_smem_desc_sw128(sbh + kk * 2048, 64 * P_BK * 2, 1024)
                                       : make_smem_desc_sw128(sbh + kk * 32, 16, 1024);
              umma_f16_pair(d_tmem, ad, bd, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            issued = true;
          }
          if (!ok) break;
          umma_commit_pair(&empty[stage]);
          if (++stage == P_STAGES) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[s0]);
#pragma unroll
        for (int h = 0; h < SPT; ++h) empty_bits ^= 1u << (s0 + h);
        if (SPT == 1) acc = acc + 1 == P_SLOTS ? 0 : acc + 1;
        const int cs = seq % P_CLC_SLOTS;
        if (!mbar_wait_bounded(&clc_full[cs], static_cast<uint32_t>(seq / P_CLC_SLOTS) & 1u, kDevErrWaitTimeoutFull,
                               abort_flag))
          break;
        int next = 0;
        const bool more = clc_next_pair_tile(clc_resp + cs * 16, p.num_tiles, next);
        mbar_arrive(&clc_empty[cs]);
        if (!more) break;
      }
      if (!ok && issued) {
        umma_commit_pair(drain);
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
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int row_in_tile = 32 * q + lane;
    unsigned char* const stage_base = smem + L::OFF_C + (warp - 2) * 2 * L::C_STAGE;  // two buffers
    int acc = 0;             // first TMEM slot of the tile (rotates when SPT == 1)
    uint32_t full_bits = 0;  // bit s: parity of slot s's next acc_full phase
    int sbuf = 0;
    const T* Cin = static_cast<const T*>(p.C_in);
    int t = pair;
    for (int seq = 0;; ++seq) {
      int b, mt, nt;
      pair_tile_coords(t, p, b, mt, nt);
      const int m0 = mt * 2 * P_BM + static_cast<int>(rank) * P_BM;
      const int n0 = nt * PBN;
      const int s0 = SPT == 1 ? acc : 0;
      if (!mbar_wait_bounded(&acc_full[s0], (full_bits >> s0) & 1u, kDevErrWaitTimeoutAccFull, abort_flag)) break;
      tc_fence_after_sync();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(s0 * P_SLOT_COLS);
      const int64_t grow = static_cast<int64_t>(m0) + row_in_tile;
#pragma unroll 1
      for (int ch = 0; ch < PBN / P_CHUNK; ++ch) {
        // Chunk ch is TMEM columns [64ch, 64ch+64) of the tile's slots.
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + ch * P_CHUNK, r0);
        tmem_ld_32x32b_x32(t_row + ch * P_CHUNK + 32, r1);
        tmem_wait_ld();
        if (ch % CHUNKS_PER_SLOT == CHUNKS_PER_SLOT - 1) {
          // Last read of this slot: the MMA issuer may overwrite it.
          tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(map_to_rank(&acc_empty[s0 + ch / CHUNKS_PER_SLOT], 0));
        }
        float v[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(r0[i]);
          v[32 + i] = __uint_as_float(r1[i]);
        }
        if (p.beta != 0.f && grow < p.M) {
          const int64_t gcol0 = static_cast<int64_t>(n0) + ch * P_CHUNK;
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
          const int64_t gcol0 = static_cast<int64_t>(n0) + ch * P_CHUNK;
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (gcol0 + i < p.N) v[i] = apply_epilogue<T>(v[i], p.bias, gcol0 + i, p.epi);
        }
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        unsigned char* sbase = stage_base + sbuf * L::C_STAGE;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 w;
          w.x = pack2_pair<T>(v[8 * j + 0], v[8 * j + 1]);
          w.y = pack2_pair<T>(v[8 * j + 2], v[8 * j + 3]);
          w.z = pack2_pair<T>(v[8 * j + 4], v[8 * j + 5]);
          w.w = pack2_pair<T>(v[8 * j + 6], v[8 * j + 7]);
          *reinterpret_cast<uint4*>(sbase + lane * 128 + ((j ^ (lane & 7)) << 4)) = w;
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmC, sbase, n0 + ch * P_CHUNK, m0 + 32 * q, b);
          bulk_commit_group();
        }
        if (p.npeers > 0) {
          // Same 32 x 64 chunk to every peer's output: lanes 8r..8r+7 write
          // the 128 contiguous bytes of one row, so each warp store is four
          // full 128-byte lines over NVLink.  Rows past M and 16-byte
          // column groups past N are skipped (N is a multiple of 8).
          const int c16 = lane & 7;
          const int64_t gcol = static_cast<int64_t>(n0) + ch * P_CHUNK + 8 * c16;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = 4 * i + (lane >> 3);
            const int64_t grow_r = static_cast<int64_t>(m0) + 32 * q + r;
            const uint4 w = *reinterpret_cast<const uint4*>(sbase + r * 128 + ((c16 ^ (r & 7)) << 4));
            if (grow_r < p.M && gcol < p.N) {
              const int64_t off = grow_r * p.ldc + gcol;
#pragma unroll
              for (int d = 0; d < P_MAX_PEERS; ++d)  // constant indices keep peer_C in the param bank
                if (d < p.npeers) *reinterpret_cast<uint4*>(static_cast<T*>(p.peer_C[d]) + off) = w;
            }
          }
        }
        sbuf ^= 1;
      }
      full_bits ^= 1u << s0;
      if (SPT == 1) acc = acc + 1 == P_SLOTS ? 0 : acc + 1;
      const int cs = seq % P_CLC_SLOTS;
      const uint32_t cpar = static_cast<uint32_t>(seq / P_CLC_SLOTS) & 1u;
      const bool got = leader ? mbar_wait_bounded(&clc_full[cs], cpar, kDevErrWaitTimeoutAccFull, abort_flag)
                              : mbar_wait_cluster_bounded(&clc_full[cs], cpar, kDevErrWaitTimeoutAccFull, abort_flag);
      if (!got) break;
      int next = 0;
      const bool more = clc_next_pair_tile(clc_resp + cs * 16, p.num_tiles, next);
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(&clc_empty[cs], 0));
      if (!more) break;
      t = next;
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
    // Peer stores of this thread are ordered before anything the stream
    // runs after the kernel (the peer barrier's release).
    if (p.npeers > 0) __threadfence_system();
  }

  tc_fence_before_sync();
  __syncthreads();
  cluster_sync_all();  // the peer is done with this CTA's smem, barriers and TMEM
  if (warp == 1) {
    tc_fence_after_sync();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(P_TMEM_COLS)
                 : "memory");
  }
}

template <typename T, bool A_MN, bool B_MN, int PBN>
int launch_tc2(const GemmProblem& p, cudaStream_t stream, const char* name, void* const* peers = nullptr,
               int npeers = 0) {
  using L = PairSmem<PBN>;
  constexpr int P_SLOT_COLS = PairCfg<PBN>::SLOT;
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mA, mB, mC;
  bool ok = true;
  if (A_MN) ok &= make_map(&mA, dt, p.A, p.M, p.K, p.batch, p.lda, p.strideA, 64, P_BK);
  else ok &= make_map(&mA, dt, p.A, p.K, p.M, p.batch, p.lda, p.strideA, P_BK, P_BM);
  if (B_MN) ok &= make_map(&mB, dt, p.B, p.N, p.K, p.batch, p.ldb, p.strideB, 64, P_BK);
  else ok &= make_map(&mB, dt, p.B, p.K, p.N, p.batch, p.ldb, p.strideB, P_BK, P_SLOT_COLS / 2);
  ok &= make_map(&mC, dt, p.C, p.N, p.M, p.batch, p.ldc, p.strideC, P_CHUNK, 32);
  if (!ok) return CUOPX_CUDA_ERROR;
  PairParams prm;
  prm.M = static_cast<int>(p.M);
  prm.N = static_cast<int>(p.N);
  prm.K = static_cast<int>(p.K);
  prm.batch = static_cast<int>(p.batch);
  prm.tiles_m = static_cast<int>((p.M + 2 * P_BM - 1) / (2 * P_BM));
  prm.tiles_n = static_cast<int>((p.N + PBN - 1) / PBN);
  prm.num_tiles = prm.tiles_m * prm.tiles_n * prm.batch;
  prm.k_blocks = static_cast<int>((p.K + P_BK - 1) / P_BK);
  prm.alpha = static_cast<float>(p.alpha);
  prm.beta = static_cast<float>(p.beta);
  prm.C_in = p.C;
  prm.ldc = p.ldc;
  prm.strideC = p.strideC;
  prm.bias = p.bias;
  prm.epi = p.epi;
  if (npeers < 0 || npeers > P_MAX_PEERS) return CUOPX_INVALID_ARGUMENT;
  prm.npeers = npeers;
  for (int i = 0; i < P_MAX_PEERS; ++i) prm.peer_C[i] = i < npeers ? peers[i] : nullptr;
  auto kern = gemm_tc2_kernel<T, A_MN, B_MN, PBN>;
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CUOPX_CUDA_ERROR;
  if (!attr_set[dev].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess)
      return CUOPX_CUDA_ERROR;
    attr_set[dev].store(true, std::memory_order_relaxed);
  }
  // One cluster per pair tile; running clusters take over unlaunched ones.
  const cudaError_t lerr = launch_pdl(kern, dim3(static_cast<unsigned>(prm.num_tiles * 2)), dim3(P_THREADS), L::ALLOC,
                                     stream, mA, mB, mC, prm);
  if (lerr != cudaSuccess) {
    cudaGetLastError();
    return cuda_failure(lerr);
  }
  note_launch(name);
  return check_launch();
}

}  // namespace

bool gemm_tc2_wanted(const GemmProblem& p) {
  // Pair tiles halve shared-memory operand traffic per FLOP, which pays off
  // over long K loops.  Measured on B200 against the 1-SM 128 x 256 kernel:
  // 256 x 512 pair tiles win from K = 4096 once there are about as many of
  // them as SM pairs (e.g. 1024 x 8192 x 4096: 50.7 vs 53.7 us), 256 x 256
  // pair tiles from K ~ 8192 with 64 tiles; at K = 1024 the 1-SM kernel,
  // whose epilogue overlaps better, is faster.
  if (!gemm_tc_supported(p)) return false;
  if (p.M < 256 || p.N < 256 || p.K < 256) return false;
  const int64_t rows = (p.M + 255) / 256;
  const int64_t tiles256 = rows * ((p.N + 255) / 256) * p.batch;
  const int64_t tiles512 = rows * ((p.N + 511) / 512) * p.batch;
  const int pairs = device_sm_count() / 2;
  return (p.K >= 4096 && p.N >= 512 && tiles512 >= (pairs * 3) / 4) || (p.K >= 6144 && tiles256 >= 64) ||
         (p.K >= 4096 && tiles256 >= 512);
}

int gemm_tc2(const GemmProblem& p, cudaStream_t stream, int pbn) { return gemm_tc2_peers(p, nullptr, 0, stream, pbn); }

namespace {

template <int PBN>
int launch_tc2_layout(const GemmProblem& p, void* const* peers, int npeers, cudaStream_t stream) {
  const bool a_mn = p.transA, b_mn = !p.transB;
  const char* name = PBN == 512   ? (npeers > 0 ? "gemm_tc2_256x512_peer" : "gemm_tc2_256x512")
                     : PBN == 256 ? (npeers > 0 ? "gemm_tc2_256x256_peer" : "gemm_tc2_256x256")
                                  : (npeers > 0 ? "gemm_tc2_256x128_peer" : "gemm_tc2_256x128");
  if (p.dtype == CUOPX_BF16) {
    if (!a_mn && b_mn) return launch_tc2<__nv_bfloat16, false, true, PBN>(p, stream, name, peers, npeers);
    if (!a_mn && !b_mn) return launch_tc2<__nv_bfloat16, false, false, PBN>(p, stream, name, peers, npeers);
    if (a_mn && b_mn) return launch_tc2<__nv_bfloat16, true, true, PBN>(p, stream, name, peers, npeers);
    return launch_tc2<__nv_bfloat16, true, false, PBN>(p, stream, name, peers, npeers);
  }
  if (!a_mn && b_mn) return launch_tc2<__half, false, true, PBN>(p, stream, name, peers, npeers);
  if (!a_mn && !b_mn) return launch_tc2<__half, false, false, PBN>(p, stream, name, peers, npeers);
  if (a_mn && b_mn) return launch_tc2<__half, true, true, PBN>(p, stream, name, peers, npeers);
  return launch_tc2<__half, true, false, PBN>(p, stream, name, peers, npeers);
}

}  // namespace

int gemm_tc2_pick_width(const GemmProblem& p, bool peers) {
  if (p.N < 512) return 256;
  const int64_t pairs = device_sm_count() / 2;
  const int64_t rows = (p.M + 255) / 256;
  const int64_t tiles256 = rows * ((p.N + 255) / 256) * p.batch;
  const int64_t tiles512 = rows * ((p.N + 511) / 512) * p.batch;
  // With peer stores the epilogue of a tile is several times longer, and
  // only the double-buffered 256 x 256 tiles overlap it with the next
  // tile's MMAs (measured on 2 B200s, C3 8192^3 column-sharded: 0.419 ms
  // with 256 x 256 tiles, 0.494 ms with 256 x 512 tiles).
  if (peers) return 256;
  // Otherwise by waves of pair tiles: a 256 x 512 tile takes twice as long
  // as a 256 x 256 one less ~5 % (fewer operand bytes from L2, measured),
  // so it wins when 2 * 0.95 * waves512 <= waves256.
  const int64_t w256 = (tiles256 + pairs - 1) / pairs;
  const int64_t w512 = (tiles512 + pairs - 1) / pairs;
  return 2 * w512 * 19 <= w256 * 20 ? 512 : 256;
}

int gemm_tc2_peers(const GemmProblem& p, void* const* peers, int npeers, cudaStream_t stream, int pbn) {
  if (pbn == 0) pbn = gemm_tc2_pick_width(p, npeers > 0);
  if (pbn == 128) return launch_tc2_layout<128>(p, peers, npeers, stream);
  return pbn == 512 ? launch_tc2_layout<512>(p, peers, npeers, stream)
                    : launch_tc2_layout<256>(p, peers, npeers, stream);
}

}  // namespace cuopx
