// Shared device/host helpers for the cuopx kernels (sm_100a only).
//
// Everything here is hand-written against the public PTX ISA: mbarrier,
// cp.async.bulk.tensor (TMA), tcgen05 (TMEM alloc / mma / ld / commit).
// Every wait loop is bounded: on expiry it records an error code in the
// module-wide device error word and returns false, so a broken pipeline
// ends the kernel with a readable status instead of hanging the GPU.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <atomic>
#include <cstdint>
#include <utility>

#include "cuopx.h"

namespace cuopx {

// ---------------------------------------------------------------------------
// Device error word.  0 = clean.  Kernels only ever CAS 0 -> code, so the
// first failure is the one reported.  Read/cleared through the C-ABI
// (cuopx_get_device_error / cuopx_clear_device_error).  Defined here: the
// device code is a single translation unit (cuopx_unity.cu).
// ---------------------------------------------------------------------------
__device__ int g_device_error = 0;

enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrWaitTimeoutFull = 1,      // consumer waited too long for a TMA stage
  kDevErrWaitTimeoutEmpty = 2,     // producer waited too long for a free stage
  kDevErrWaitTimeoutAccFull = 3,   // epilogue waited too long for the accumulator
  kDevErrWaitTimeoutAccEmpty = 4,  // MMA waited too long for the epilogue
  kDevErrWaitTimeoutStore = 5,     // bulk store drain took too long
  kDevErrSplitReduce = 6,          // split-K arrival counter out of range
  kDevErrAbortDrain = 7,           // in-flight TMA did not land during abort
  kDevErrPeerTimeout = 8,          // a peer GPU did not reach the barrier
  kDevErrSchedule = 9,             // launch-control answer outside the grid
};

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// Wall-clock bound for any single wait: 1 s of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// First 1024-byte boundary (swizzle-atom alignment) at or after `raw`, a
// shared-memory array.  The offset is computed from the shared-window
// address and added to the array pointer, so the compiler still knows the
// result is shared memory and emits shared (not generic) loads and stores.
__device__ __forceinline__ unsigned char* align_smem_1024(unsigned char* raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel on its stream is still
// running; it must call grid_dependency_wait() before its first access to
// global memory that the previous kernel may write or read, which returns
// once that kernel has completed and its writes are visible.
// grid_launch_dependents() lets the next such kernel start launching once
// every CTA of this grid has called it or exited.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: launch `kernel` with programmatic stream serialization allowed.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Thread-block clusters: rank within the cluster, distributed shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

// Every thread of every CTA of the cluster arrives (release) and waits
// (acquire): shared-memory writes made before it, including remote ones, are
// visible after it.  Every thread of the cluster must execute it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `threads` threads
// (a multiple of 32; whole warps).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// The two halves of cluster_sync_all, for a barrier whose arrival comes
// early and whose wait comes much later (each thread does both, in order).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Arrival without release semantics (~1 k cycles cheaper than the release
// form, measured): for threads that publish nothing, or whose mbarrier
// initialisations were published by fence.mbarrier_init.release.cluster.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from this CTA's shared memory to `dst` in another CTA of the cluster (a
// shared::cluster address from map_to_rank); the copy completes `bytes` of
// transaction count on the mbarrier `bar` of the destination CTA (also a
// shared::cluster address).  No multicast.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Host: launch `kernel` in clusters of `cluster_x` CTAs along x, with
// programmatic stream serialization allowed.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Cluster launch control (sm_100): a running CTA asks the hardware to cancel
// a CTA of the same grid that has not been launched yet and takes over its
// work.  The 16-byte response lands in shared memory and completes 16 bytes
// on `bar` (the issuing thread posts expect_tx(16) first).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void clc_try_cancel(void* resp, uint64_t* bar) {
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
                   smem_u32(resp)),
               "r"(smem_u32(bar))
               : "memory");
}

// Decode a completed response: true and the cancelled CTA's blockIdx.x, or
// false when no unlaunched CTA was left.
__device__ __forceinline__ bool clc_query(const void* resp, int& ctaid_x) {
  uint32_t canceled, x;
  asm volatile(
      "{\n\t.reg .b128 r;\n\t.reg .pred p;\n\t"
      "ld.shared.b128 r, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r;\n\t}"
      : "=r"(canceled), "=r"(x)
      : "r"(smem_u32(resp))
      : "memory");
  ctaid_x = static_cast<int>(x);
  return canceled != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test (cluster-scope acquire) of whether the phase with the
// given parity has completed.  An MMA-issuing thread tests the next stage's
// barrier while the current stage's last MMAs are still being issued, so
// the test's latency is not a gap in the tensor pipe (a blocking wait
// between stages costs ~120 cycles of idle pipe per stage, measured on
// B200 with back-to-back tf32 MMAs).
__device__ __forceinline__ bool mbar_test_wait_cluster(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same test with CTA-scope acquire (the barrier's arrivals come from
// this CTA).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (and records `err`) after kWaitLimitNs, or immediately once another
// role has raised *abort.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int err,
                                                  volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((it & 255u) == 0u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_device_error(err);
        *abort = 1;
        return false;
      }
    }
  }
}

// Bounded wait with cluster-scope acquire (data written by the partner CTA
// before its release-arrive is visible afterwards).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, int err,
                                                          volatile int* abort) {
  const uint32_t addr = smem_u32(bar);
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 255u) == 255u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_device_error(err);
        *abort = 1;
        return false;
      }
    }
  }
}

// Arrive (release, cluster scope) on an mbarrier of any CTA of the cluster.
// The cluster-scope release orders all of this thread's prior memory
// operations and costs ~1-2k cycles; use it where the arrival publishes
// data that another CTA's threads read.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Arrive on an mbarrier of any CTA of the cluster with the default
// (CTA-scope) release: the hand-off from a CTA's converter warps to the pair
// MMA that reads their shared memory and TMEM, after the writer's
// fence.proxy.async and tcgen05.fence::before_thread_sync.  Measured on
// B200: ~100 cycles against ~1-2k for the cluster-scope release.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) — loads without any multicast qualifier.
// ---------------------------------------------------------------------------
// L2 prefetch of one TMA box (no data is returned, nothing is multicast).
__device__ __forceinline__ void tma_prefetch_3d(const void* tmap, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(tmap), "r"(c0), "r"(c1),
               "r"(c2)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (fp16 or bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A * B, kind::tf32 (fp32 containers, tf32 multiply, fp32 accumulate).
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::tf32: A is M=128 lanes (one row
// per lane) by K 32-bit columns at a_tmem.
__device__ __forceinline__ void umma_tf32_a_tmem(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair MMA (cta_group::2, issued by the even CTA of the pair), kind::tf32:
// each CTA's TMEM holds its 128 rows of A at a_tmem and its half of B's
// columns at the same shared-memory offset; D gets each CTA's 128 rows.
__device__ __forceinline__ void umma_tf32_pair_a_tmem(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                      uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (same offset) in every CTA of the cluster named by `mask`
// (bit i = CTA rank i) once all prior tcgen05 ops of this thread complete;
// issued for a pair MMA (cta_group::2).
__device__ __forceinline__ void umma_commit_pair_mask(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns from 16 registers per thread
// (the warp may address only its own lane quarter).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 op previously issued by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 32 consecutive columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (tcgen05 shared-memory matrix descriptor, 64-bit).
//   [0,14)  start address >> 4
//   [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4
//   [46,48) version = 1 (sm_100)
//   [49,52) base offset (0: swizzle atoms are 1024-byte aligned)
//   [52]    LBO mode (0)
//   [61,64) layout: 0 none, 2 = 128-byte swizzle
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// 128-byte swizzle with 16-byte atoms (layout 2): 8-row, 1024-byte atoms.
__device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                         uint32_t sbo_bytes) {
  return make_smem_desc(smem_addr, lbo_bytes, sbo_bytes, 2u);
}

// 128-byte swizzle with 32-byte atoms (layout 1): 4-row, 512-byte atoms; the
// only shared-memory layout the tensor cores take for MN-major 32-bit (tf32)
// operands.  TMA writes it with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
__device__ __forceinline__ uint64_t make_smem_desc_sw128_32b(uint32_t smem_addr, uint32_t lbo_bytes,
                                                             uint32_t sbo_bytes) {
  return make_smem_desc(smem_addr, lbo_bytes, sbo_bytes, 1u);
}

// Instruction descriptor for kind::f16 / kind::tf32 with fp32 accumulation.
//   [4,6) D format (1 = f32); [7,10) A format; [10,13) B format
//   (0 = f16, 1 = bf16, 2 = tf32); [15] A major (1 = MN-major);
//   [16] B major; [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, bool a_mn_major, bool b_mn_major, int M,
                                                  int N) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((static_cast<uint32_t>(N) >> 3) << 17) |
         ((static_cast<uint32_t>(M) >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Scalar conversion helpers shared by the SIMT kernels.
// ---------------------------------------------------------------------------
template <typename T>
struct AccOf {
  using type = float;
};
template <>
struct AccOf<double> {
  using type = double;
};

template <typename T>
__device__ __forceinline__ typename AccOf<T>::type to_acc(T v) {
  return static_cast<typename AccOf<T>::type>(v);
}
template <>
__device__ __forceinline__ float to_acc<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_acc<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_acc(typename AccOf<T>::type v) {
  return static_cast<T>(v);
}
template <>
__device__ __forceinline__ __half from_acc<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// alpha*acc + beta*c exactly as the reference's kernels compute
// `alpha * sum + beta * C` (src/cuda_op/detail/cuBlas/gemm.cu:41, gemv.cu:21):
// beta*c rounded, then one fused multiply-add with alpha*acc.  (Measured on
// B200 against the reference built from its sources: this form reproduces
// every output bit; rounding alpha*acc separately does not when alpha != 1
// and beta != 0.)  With beta == 0, C is not read: the rounded alpha*acc.
__device__ __forceinline__ float epi_axpby(float alpha, float acc, float beta, float c) {
  return __fmaf_rn(alpha, acc, __fmul_rn(beta, c));
}
__device__ __forceinline__ double epi_axpby(double alpha, double acc, double beta, double c) {
  return __fma_rn(alpha, acc, __dmul_rn(beta, c));
}
__device__ __forceinline__ float epi_scale(float alpha, float acc) { return __fmul_rn(alpha, acc); }
__device__ __forceinline__ double epi_scale(double alpha, double acc) { return __dmul_rn(alpha, acc); }

// Fused GEMM epilogue, applied to alpha*acc (+ beta*C) before the one
// rounding to the output type: + bias[col] (rounded add, never contracted
// with the product), then ReLU(x) = x if x > 0 else +0 (NaN -> +0).
__device__ __forceinline__ float epi_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double epi_add(double a, double b) { return __dadd_rn(a, b); }

template <typename T>
__device__ __forceinline__ typename AccOf<T>::type apply_epilogue(typename AccOf<T>::type v, const void* bias,
                                                                  int64_t col, int epi) {
  using Acc = typename AccOf<T>::type;
  if (epi & CUOPX_EPI_BIAS) v = epi_add(v, to_acc<T>(static_cast<const T*>(bias)[col]));
  if (epi & CUOPX_EPI_RELU) v = v > Acc(0) ? v : Acc(0);
  return v;
}

}  // namespace cuopx
