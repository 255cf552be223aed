#!/usr/bin/env python
"""Benchmark of the cuop_b200 dense BLAS hot path on B200.

Headline (one JSON line, rank 0): bf16 strided-batched GEMM, 4096 batches of
C[128x128] = A[128x64] B[64x128] (fp32 accumulate, bf16 out, inputs N(0,1)),
sharded by batch over the N ranks with no collective: rank r runs batches
[r*4096/N, (r+1)*4096/N).  The total work is fixed as N grows (strong
scaling).  One step = one batched call per rank on a fresh input set (input
sets rotated so that their total exceeds the 126 MB L2).  Metric: HBM GB/s of
algorithmic traffic (A and B read once, C written once), whole job.

`e2e` is the same workload through the per-call public API with the data in
pinned host memory: cuop_b200.batched_gemm_host streams each rank's shard
host -> device -> host every step (both PCIe directions overlapped with the
GEMMs) and returns when the host holds C.

Under "configs" the same line carries the other shapes of the path, each with
its clock record and a parity check:
  c2  fp32 GEMV 8192^2, plain + transposed (replicas at N > 1), with its own
      roofline, per-call e2e and CPU baseline;
  c1  fp32 GEMM 1024^3 (replicas);
  c3  fp16 GEMM 8192^3, column-sharded at N > 1 with the full output on
      every rank (fused peer-store epilogue, and GEMM + NCCL all-gather);
  c5  bf16 linear 4096 x 8192 x 28672, the same way.
`--configs c3,c5` (etc.) runs a subset.  At N > 1 every sharded output is
checked on every rank (complete sampled rows and columns against an fp32
product, and a checksum all-gather showing every rank holds the same bytes).

`--impl reference` times the reference path's CPU restatement (the
reference has no CPU implementation of its own) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# Headline workload (C4).
BATCH, BM, BN, BK = 4096, 128, 128, 64
C4_BYTES_PER_BATCH = (BM * BK + BK * BN + BM * BN) * 2
C4_BYTES = BATCH * C4_BYTES_PER_BATCH  # 268,435,456
GEMV_N = 8192
GEMV_BYTES = (GEMV_N * GEMV_N + 2 * GEMV_N) * 4  # A + x + y (beta = 0: y not read)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FP32_SIMT_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# Nominal B200 figures, reported beside the measured-peak fractions.
SPEC_HBM_GBS = 8000.0
SPEC_DENSE_16BIT_TFLOPS = 2250.0
LOWP_TOL = 1e-2

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernels, from the ncu captures summarised in profiles/ (file
# named beside each figure); per batch for the batched kernel.
NCU_TRAFFIC = {
    # 134.3 MB read + 78.2 MB written in one 4096-batch launch (the rest of C
    # was still dirty in L2 when the isolated launch ended)
    "gemm_tc_128x128_2cta": {"bytes_per_batch": 51874,
                             "source": "profiles/gemm_tc_128x128_2cta_bf16_batched_4096x128x128x64_ncu.md"},
    "gemv_t_lsu": {"bytes": 272088832, "source": "profiles/gemv_f32_8192_ncu.md"},
    "gemv_n_xreg": {"bytes": 272280576, "source": "profiles/gemv_f32_8192_ncu.md"},
}


# --------------------------------------------------------------------------- util
def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)) or None, \
                "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, None, "fallback"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.ok = False
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"], "samples": 0}
        reasons = [k for k, bit in self.REASONS.items() if self.reasons & bit and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


def dist_init(world):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))))
    return dist


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_gather_floats(vals, world: int):
    """Every rank's list of floats, as a list per rank (collective)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    if world == 1:
        return [t.tolist()]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def capture_graph(fn, n):
    """CUDA graph of fn(0..n-1).  The launches inside are the library's own
    kernels through its public API; replaying the graph removes the host's
    per-call Python/ctypes overhead from the device timeline.  Returns the
    graph and the number of cuopx kernels it holds."""
    import torch
    import cuop_b200 as cx

    fn(0)  # lazy per-device set-up (function attributes, workspaces) outside capture
    torch.cuda.synchronize()
    c0 = cx.launch_count()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fn(i)
    torch.cuda.synchronize()
    return g, cx.launch_count() - c0


def time_graph(fn, steps, warmup, world, align=None, clock=None):
    """Device time (ms per call) of `steps` calls of fn replayed as one CUDA
    graph after `warmup` eager calls; max over ranks.  `align`, if given, is
    launched on the stream just before the timed replay (a cross-GPU barrier,
    so that host-side skew between ranks stays out of the timed region).
    `clock` (a ClockSampler) samples the clocks during the timed replay."""
    import torch
    from contextlib import nullcontext

    for i in range(warmup):
        fn(i)
    g, launches = capture_graph(fn, steps)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The clock sampler starts (and sleeps its start-up interval) before the
    # untimed replay, so the GPU is busy right up to the timed region.
    with (clock or nullcontext()):
        g.replay()  # untimed: uploads the graph, warms clocks and caches
        barrier(world)
        if align is not None:
            align()
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    barrier(world)
    del g
    return max_over_ranks(ms, world), launches


def time_loop(fn, steps, warmup, world, clock=None):
    """Eager device time (ms per call) of `steps` calls, max over ranks (used
    where a step holds NCCL collectives, which stay out of graphs)."""
    import torch
    from contextlib import nullcontext

    for _ in range(warmup):
        fn(0)
    barrier(world)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with (clock or nullcontext()):
        e0.record(s)
        for i in range(steps):
            fn(i)
        e1.record(s)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    barrier(world)
    return max_over_ranks(ms, world)


def time_host_loop(fn, steps, warmup, world):
    """Wall time (ms per call) of `steps` host-synchronous calls, max over
    ranks: each call returns only when its results are in host memory."""
    for i in range(warmup):
        fn(i)
    barrier(world)
    t0 = time.perf_counter()
    for i in range(steps):
        fn(i)
    ms = (time.perf_counter() - t0) * 1e3 / steps
    barrier(world)
    return max_over_ranks(ms, world)


def fp32_product(a, b):
    """Plain fp32 product (TF32 off) of widened operands on the GPU: the
    reference for full-size checks, where the CPU oracle would take minutes."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a.float() @ b.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def max_rel(got, ref) -> float:
    """max|C - R| / max|R| (the fp16/bf16 bound is 1e-2)."""
    den = float(ref.abs().max())
    return float((got.float() - ref).abs().max()) / (den if den > 0 else 1.0)


def checksum(t) -> list:
    """Two position-weighted sums of a 2-D 16-bit tensor's bit patterns (row-
    and column-weighted): equal on two ranks only if the bytes agree, with
    overwhelming probability."""
    import torch

    v = t.contiguous().view(torch.int16).to(torch.int64)
    rows = v.sum(dim=1)
    cols = v.sum(dim=0)
    wr = torch.arange(1, rows.numel() + 1, device=v.device, dtype=torch.int64)
    wc = torch.arange(1, cols.numel() + 1, device=v.device, dtype=torch.int64)
    return [float(int((rows * wr).sum()) % (1 << 52)), float(int((cols * wc).sum()) % (1 << 52))]


# --------------------------------------------------------------------------- C4 (headline)
def c4_inputs(dev, lb, seed):
    import torch

    per_set = lb * C4_BYTES_PER_BATCH
    sets = max(2, math.ceil(400e6 / per_set))  # > 3x the 126 MB L2
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    As = [torch.randn(lb, BM, BK, device=dev, generator=g).bfloat16() for _ in range(sets)]
    Bs = [torch.randn(lb, BK, BN, device=dev, generator=g).bfloat16() for _ in range(sets)]
    Cs = [torch.empty(lb, BM, BN, device=dev, dtype=torch.bfloat16) for _ in range(sets)]
    return As, Bs, Cs, sets


def c4_parity(As, Bs, Cs, world):
    """Each rank's shard against an fp32 product on 16 sampled batches of the
    last rotation set computed; max over ranks."""
    import torch

    lb = As[0].size(0)
    g = torch.Generator().manual_seed(5)
    idx = sorted(set([0, lb - 1] + torch.randint(0, lb, (14,), generator=g).tolist()))
    k = 0
    err = 0.0
    for b in idx:
        ref = fp32_product(As[k][b], Bs[k][b])
        err = max(err, max_rel(Cs[k][b], ref))
    return {"max_rel": max_over_ranks(err, world), "tol": LOWP_TOL, "batches_checked_per_rank": len(idx),
            "reference": "fp32 product (TF32 off) of the same bf16 inputs"}


def run_c4(args, rank, world, local_rank):
    import torch
    import cuop_b200 as cx
    from cuop_b200 import sharding

    dev = torch.device("cuda", local_rank)
    b0, b1 = sharding.shard_range(BATCH, rank, world)
    lb = b1 - b0
    As, Bs, Cs, sets = c4_inputs(dev, lb, seed=1000 + rank)

    def step(i):
        cx.batched_gemm(As[i % sets], Bs[i % sets], Cs[i % sets])

    for i in range(args.warmup):
        step(i)
    barrier(world)
    K = args.steps
    g_step, launches = capture_graph(step, K)
    kname = cx.last_kernel()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    # The sampler starts before the untimed replay (its start-up sleep would
    # otherwise leave the GPU idle right before the timed region).
    with ClockSampler(local_rank) as clk:
        g_step.replay()  # untimed: uploads the graph, warms clocks and caches
        barrier(world)
        e0.record(stream)
        g_step.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1) / K
    del g_step
    barrier(world)
    ms = max_over_ranks(ms_local, world)
    for k in range(sets):  # outputs of every set, for the parity check below
        cx.batched_gemm(As[k], Bs[k], Cs[k])
    parity = c4_parity(As, Bs, Cs, world)

    hbm, _, _, peak_src = load_peaks()
    value = C4_BYTES / (ms * 1e-3) / 1e9
    local_bytes = lb * C4_BYTES_PER_BATCH
    achieved = local_bytes / (ms_local * 1e-3) / 1e9  # one launch per step on this rank
    tr = NCU_TRAFFIC.get(kname, {})
    traffic = tr["bytes_per_batch"] * lb if tr.get("bytes_per_batch") else None
    line = {
        "metric": "bf16 batched GEMM 4096 x (128x128x64), batch-sharded: HBM GB/s", "value": round(value, 2),
        "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "bf16 strided-batched GEMM C[b] = A[b] B[b], batch 4096, M=N=128, K=64, "
                               "A,B ~ N(0,1), fp32 accumulate, bf16 out", "global_batch": BATCH,
                   "per_gpu_batch": lb, "parallelism": f"batch-sharded x{world}, no collective",
                   "l2": f"inputs larger than L2: {sets} rotated input sets of {local_bytes / 1e6:.1f} MB per rank",
                   "bytes_per_step": C4_BYTES},
        "roofline": {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1), "peak": hbm,
                     "peak_source": f"{peak_src} hbm_gbs (burst copy)", "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "frac_spec": round(achieved / SPEC_HBM_GBS, 4),
                     "spec_peak": SPEC_HBM_GBS, "traffic": traffic, "traffic_source": tr.get("source"),
                     "algorithmic_bytes": local_bytes, "per": "one launch on one GPU"},
        "gpu_launches": launches,
        "timing": "timed region = one CUDA graph replay of K steps (one batched launch per rank each)",
        "clocks": clk.summary(),
        "parity": parity,
    }
    line["e2e"] = c4_e2e(args, rank, world, local_rank, lb)
    del As, Bs, Cs
    torch.cuda.empty_cache()
    return line


def c4_e2e(args, rank, world, local_rank, lb):
    """The same workload through the per-call public API with the data in
    pinned host memory: every step, cuop_b200.batched_gemm_host copies this
    rank's A and B shard in, runs the batched GEMM and copies C out (copies of
    both directions overlapped with the GEMMs), returning when the host holds
    C.  Two host input sets alternate.  Checked bit for bit against the device
    call on the same inputs."""
    import torch
    import cuop_b200 as cx

    dev = torch.device("cuda", local_rank)
    g = torch.Generator().manual_seed(77 + rank)
    hA = [torch.randn(lb, BM, BK, generator=g).bfloat16().pin_memory() for _ in range(2)]
    hB = [torch.randn(lb, BK, BN, generator=g).bfloat16().pin_memory() for _ in range(2)]
    hC = torch.empty(lb, BM, BN, dtype=torch.bfloat16).pin_memory()

    cx.batched_gemm_host(hA[0], hB[0], hC)
    dC = cx.batched_gemm(hA[0].to(dev), hB[0].to(dev))
    torch.cuda.synchronize()
    if not torch.equal(hC, dC.cpu()):
        raise RuntimeError("batched_gemm_host result differs from the device call")
    del dC

    steps = max(5, min(args.steps, 50))
    ms = time_host_loop(lambda i: cx.batched_gemm_host(hA[i % 2], hB[i % 2], hC), steps, 3, world)
    return {"value": round(C4_BYTES / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": world * lb * (BM * BK + BK * BN) * 2,
            "d2h_bytes_per_step": world * lb * BM * BN * 2, "per_rank_h2d_bytes": lb * (BM * BK + BK * BN) * 2,
            "ms_per_step": round(ms, 4), "steps": steps,
            "path": "cuop_b200.batched_gemm_host per step (one call per rank): pinned host A,B shard -> device in "
                    "chunks, cuopx_gemm_strided_batched per chunk, C -> pinned host, host waits; wall clock, "
                    "max over ranks"}


# --------------------------------------------------------------------------- CPU baselines (oracle)
def _timed(fn, budget_s, max_reps=20):
    fn()  # page-in
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= max_reps:
            return el / reps


def cpu_c4_baseline(budget_s: float = 3.0):
    """The oracle's batched bf16 GEMM (CPU restatement of the reference's
    batched kernel arithmetic) on the C4 workload: all host threads on the
    full 4096 batches, and one thread on a 256-batch slab."""
    import oracle as O

    nt = O.threads()
    A = O.to_lowp(O.normal((BATCH, BM, BK), seed=4), O.BF16)
    B = O.to_lowp(O.normal((BATCH, BK, BN), seed=5), O.BF16)
    t = _timed(lambda: O.gemm_batched_lowp(O.BF16, A, B, nthreads=nt), budget_s)
    slab = 256
    t1 = _timed(lambda: O.gemm_batched_lowp(O.BF16, A[:slab], B[:slab], nthreads=1), budget_s)
    return {"value": round(C4_BYTES / t / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"full workload, 4096 x 128x128x64 bf16 batched GEMM in {t * 1e3:.0f} ms, oracle/cpu_ref.c, "
                      f"OpenMP {nt} threads",
            "single_thread": {"value": round(slab * C4_BYTES_PER_BATCH / t1 / 1e9, 3), "unit": "GB/s", "cores": 1,
                              "sample": f"{slab}-batch slab in {t1 * 1e3:.0f} ms"},
            "cpu_model": cpu_model()}


def cpu_gemv_baseline(budget_s: float = 3.0):
    """The CPU restatement of the reference GEMV on all host threads (full
    8192^2 plain + transposed) and on one thread (a 512-row slab)."""
    import oracle as O

    nt = O.threads()
    A = O.uniform((GEMV_N, GEMV_N), seed=0)
    x = O.uniform(GEMV_N, seed=1)
    t = _timed(lambda: (O.gemv_f32(A, x, nthreads=nt), O.gemv_f32(A, x, trans=True, nthreads=nt)), budget_s, 50)
    rows = 512
    As, xs = A[:rows], x[:rows]
    t1 = _timed(lambda: (O.gemv_f32(As, x, nthreads=1), O.gemv_f32(As, xs, trans=True, nthreads=1)), budget_s, 50)
    slab_bytes = 2 * (rows * GEMV_N + GEMV_N + rows) * 4
    return {"value": round(2 * GEMV_BYTES / t / 1e9, 2), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"full workload, plain + transposed fp32 GEMV 8192^2 in {t * 1e3:.0f} ms, oracle/cpu_ref.c, "
                      f"OpenMP {nt} threads",
            "single_thread": {"value": round(slab_bytes / t1 / 1e9, 3), "unit": "GB/s", "cores": 1,
                              "sample": f"{rows}-row slab, plain + transposed, {t1 * 1e3:.0f} ms"},
            "cpu_model": cpu_model()}


def cpu_config_baselines(budget_s: float = 1.5) -> dict:
    """The oracle on the GEMM configs, all host threads and one thread: C1 in
    full (one thread: a 128-row slab), C3 and C5 on a 64-row slab of A (one
    thread: 8 rows), full-problem times extrapolated by rows."""
    import oracle as O

    nt = O.threads()
    out = {}
    n = 1024
    A, B = O.uniform((n, n), seed=0), O.uniform((n, n), seed=1)
    t = _timed(lambda: O.gemm_f32(A, B, nthreads=nt), budget_s)
    t1 = _timed(lambda: O.gemm_f32(A[:128], B, nthreads=1), budget_s)
    out["c1_fp32_gemm_1024"] = {
        "value": round(2 * n ** 3 / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt, "kind": "port",
        "sample": f"full 1024^3 fp32 GEMM, {t * 1e3:.1f} ms",
        "single_thread": {"value": round(2 * 128 * n * n / t1 / 1e12, 4), "unit": "TFLOP/s",
                          "sample": f"128-row slab, {t1 * 1e3:.1f} ms"}}
    n, rows, rows1 = 8192, 64, 8
    A = O.to_lowp(O.normal((rows, n), seed=2) / math.sqrt(n), O.F16)
    B = O.to_lowp(O.normal((n, n), seed=3) / math.sqrt(n), O.F16)
    t = _timed(lambda: O.gemm_lowp(O.F16, A, B, nthreads=nt), budget_s)
    t1 = _timed(lambda: O.gemm_lowp(O.F16, A[:rows1], B, nthreads=1), budget_s, 3)
    out["c3_fp16_gemm_8192"] = {
        "value": round(2 * rows * n * n / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt, "kind": "port",
        "sample": f"64-row slab of the 8192^3 fp16 GEMM, {t * 1e3:.0f} ms; extrapolated full problem "
                  f"{t * n / rows:.1f} s",
        "single_thread": {"value": round(2 * rows1 * n * n / t1 / 1e12, 5), "unit": "TFLOP/s",
                          "sample": f"{rows1}-row slab, {t1 * 1e3:.0f} ms; extrapolated {t1 * n / rows1:.0f} s"}}
    M, K, N_ = 4096, 8192, 28672
    X = O.to_lowp(O.normal((rows, K), seed=6), O.BF16)
    W = O.to_lowp(O.normal((K, N_), seed=7) * 0.02, O.BF16)
    t = _timed(lambda: O.gemm_lowp(O.BF16, X, W, nthreads=nt), budget_s)
    t1 = _timed(lambda: O.gemm_lowp(O.BF16, X[:rows1], W, nthreads=1), budget_s, 3)
    out["c5_bf16_linear_4096x8192x28672"] = {
        "value": round(2 * rows * K * N_ / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt, "kind": "port",
        "sample": f"64-row slab of the 4096 x 8192 x 28672 bf16 GEMM, {t * 1e3:.0f} ms; extrapolated full problem "
                  f"{t * M / rows:.1f} s",
        "single_thread": {"value": round(2 * rows1 * K * N_ / t1 / 1e12, 5), "unit": "TFLOP/s",
                          "sample": f"{rows1}-row slab, {t1 * 1e3:.0f} ms; extrapolated {t1 * M / rows1:.0f} s"}}
    return out


# --------------------------------------------------------------------------- C2 GEMV
def gemv_inputs(dev, sets: int, seed: int = 0):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    An = [torch.rand(GEMV_N, GEMV_N, device=dev, generator=g).mul_(2).sub_(1) for _ in range(sets)]
    At = [torch.rand(GEMV_N, GEMV_N, device=dev, generator=g).mul_(2).sub_(1) for _ in range(sets)]
    x = torch.rand(GEMV_N, device=dev, generator=g).mul_(2).sub_(1)
    return An, At, x


def run_gemv(args, rank, world, local_rank):
    """C2: plain + transposed fp32 GEMV 8192^2 per step (replicas at N > 1)."""
    import torch
    import cuop_b200 as cx

    dev = torch.device("cuda", local_rank)
    sets = 2
    An, At, x = gemv_inputs(dev, sets, seed=1234 + rank)
    yn = torch.empty(GEMV_N, device=dev)
    yt = torch.empty(GEMV_N, device=dev)

    def step(i):
        cx.gemv(An[i % sets], x, yn)
        cx.gemv(At[i % sets], x, yt, trans=True)

    K = max(20, min(args.steps, 2000))
    clk = ClockSampler(local_rank)
    ms, launches = time_graph(step, K, max(3, args.warmup), world, clock=clk)
    cx.gemv(An[0], x, yn)
    kn = cx.last_kernel()
    cx.gemv(At[0], x, yt, trans=True)
    kt = cx.last_kernel()
    # Per-kernel device time: each kernel alone, back to back, same rotation.
    t_n, _ = time_graph(lambda i: cx.gemv(An[i % sets], x, yn), K, 2, world)
    t_t, _ = time_graph(lambda i: cx.gemv(At[i % sets], x, yt, trans=True), K, 2, world)
    # Parity: both results against an fp64-accumulated product on the GPU.
    ref_n = (An[0].double() @ x.double())
    ref_t = (At[0].double().t() @ x.double())
    cx.gemv(An[0], x, yn)
    cx.gemv(At[0], x, yt, trans=True)
    rel = max(float((yn.double() - ref_n).norm() / ref_n.norm()), float((yt.double() - ref_t).norm() / ref_t.norm()))

    hbm, _, _, peak_src = load_peaks()
    dom_name, dom_ms = (kt, t_t) if t_t >= t_n else (kn, t_n)
    achieved = GEMV_BYTES / (dom_ms * 1e-3) / 1e9
    kernels = {k: {"ms": round(t, 5), "gbs": round(GEMV_BYTES / (t * 1e-3) / 1e9, 1),
                   "frac": round(GEMV_BYTES / (t * 1e-3) / 1e9 / hbm, 4)} for k, t in ((kn, t_n), (kt, t_t))}
    tr = NCU_TRAFFIC.get(dom_name, {})
    out = {
        "gbs_total": round(world * 2 * GEMV_BYTES / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 5),
        "workload": "fp32 GEMV y=1.0*A*x+0.0*y, M=N=8192, plain + transposed, A,x ~ U[-1,1); 2 matrix sets "
                    "per kind rotated (1 GiB > L2)",
        "parallelism": f"replicas x{world} (GEMV does not shard)",
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1), "peak": hbm,
                     "peak_source": f"{peak_src} hbm_gbs (burst copy)", "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "frac_spec": round(achieved / SPEC_HBM_GBS, 4),
                     "traffic": tr.get("bytes"), "traffic_source": tr.get("source"),
                     "algorithmic_bytes": GEMV_BYTES},
        "kernels": kernels, "gpu_launches": launches, "clocks": clk.summary(),
        "parity": {"rel_frobenius_max": max_over_ranks(rel, world), "tol": 1e-5 * math.sqrt(GEMV_N),
                   "reference": "fp64 product on the GPU"},
    }
    out["e2e"], out["e2e_graph_replay"] = gemv_e2e(args, rank, world, local_rank, An, At)
    del An, At
    torch.cuda.empty_cache()
    return out


def gemv_e2e(args, rank, world, local_rank, An, At):
    """The GEMV through the public API in the plugin's usage model
    (GemvJITPlugin holds the matrix as its weight, set once and resident;
    each Execute takes x and returns y).  Per step: cuop_b200.copy brings a
    fresh x from pinned host memory (the copy kernel reads the pinned
    buffer), both cuop_b200.gemv calls write y straight into pinned host
    memory, and the host waits.  Timed as three ordinary calls per step
    (`e2e`) and, for comparison, with the three launches replayed as one CUDA
    graph (`e2e_graph_replay`)."""
    import torch
    import cuop_b200 as cx

    dev = torch.device("cuda", local_rank)
    sets = len(An)
    g = torch.Generator().manual_seed(77 + rank)
    hx = [(torch.rand(GEMV_N, generator=g) * 2 - 1).pin_memory() for _ in range(sets)]
    hy = torch.empty(2, GEMV_N, pin_memory=True)
    dx = torch.empty(GEMV_N, device=dev)
    stream = torch.cuda.current_stream()

    def body(k):
        cx.copy(hx[k], dx)
        cx.gemv(An[k], dx, hy[0])
        cx.gemv(At[k], dx, hy[1], trans=True)

    # The host copy of the results is the device's answer.
    yn = torch.empty(GEMV_N, device=dev)
    yt = torch.empty(GEMV_N, device=dev)
    body(0)
    stream.synchronize()
    cx.gemv(An[0], dx, yn)
    cx.gemv(At[0], dx, yt, trans=True)
    torch.cuda.synchronize()
    if not (torch.equal(hy[0], yn.cpu()) and torch.equal(hy[1], yt.cpu())):
        raise RuntimeError("GEMV results in pinned host memory differ from the device results")

    def step(i):
        body(i % sets)
        stream.synchronize()  # the host has the step's results

    steps = max(5, min(args.steps, 500))
    ms = time_host_loop(step, steps, 5, world)

    graphs = []
    for k in range(sets):
        body(k)
        torch.cuda.synchronize()
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gk):
            body(k)
        graphs.append(gk)

    def gstep(i):
        graphs[i % sets].replay()
        stream.synchronize()

    ms_g = time_host_loop(gstep, steps, 5, world)
    del graphs
    common = {"unit": "GB/s", "h2d_bytes_per_step": world * GEMV_N * 4, "d2h_bytes_per_step": world * 2 * GEMV_N * 4,
              "steps": steps}
    e2e = {"value": round(world * 2 * GEMV_BYTES / (ms * 1e-3) / 1e9, 2), "ms_per_step": round(ms, 4), **common,
           "path": "per step: cuop_b200.copy (x from pinned host) + 2 x cuop_b200.gemv (y into pinned host), "
                   "three ordinary calls, then host synchronisation; wall clock, max over ranks"}
    e2e_g = {"value": round(world * 2 * GEMV_BYTES / (ms_g * 1e-3) / 1e9, 2), "ms_per_step": round(ms_g, 4),
             **common, "path": "the same three launches replayed as one CUDA graph per step, then host "
                               "synchronisation"}
    return e2e, e2e_g


# --------------------------------------------------------------------------- other configs
def run_configs(args, rank, world, local_rank):
    import torch
    import cuop_b200 as cx
    from cuop_b200 import sharding

    dev = torch.device("cuda", local_rank)
    hbm, bf16_peak, bf16_sus, peak_src = load_peaks()
    out = {}
    steps = max(5, min(args.steps, 30))
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)

    want = {c.strip().lower() for c in args.configs.split(",") if c.strip()}
    if "c2" in want:
        out["c2_fp32_gemv_8192"] = run_gemv(args, rank, world, local_rank)
    if "c1" in want:
        out.update(_config_c1(cx, dev, g, steps, world, local_rank))
    if "c3" in want:
        out.update(_config_c3(cx, sharding, dev, steps, rank, world, local_rank, bf16_peak, peak_src))
    if "c5" in want:
        out.update(_config_c5(cx, sharding, dev, steps, rank, world, local_rank, bf16_peak))
    return out


def _config_c1(cx, dev, g, steps, world, local_rank):
    """fp32 GEMM 1024^3 (replicas), default mode (3xTF32 on the tensor cores)."""
    import torch

    n = 1024
    A = torch.rand(n, n, device=dev, generator=g) * 2 - 1
    B = torch.rand(n, n, device=dev, generator=g) * 2 - 1
    C = torch.empty(n, n, device=dev)
    clk = ClockSampler(local_rank)
    ms, launches = time_graph(lambda i: cx.gemm(A, B, C), steps * 20, 5, world, clock=clk)
    kname = cx.last_kernel()
    ref = (A.double() @ B.double())
    cx.gemm(A, B, C)
    rel = float((C.double() - ref).norm() / ref.norm())
    tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
    return {"c1_fp32_gemm_1024": {"tflops_total": round(world * tf, 3), "ms": round(ms, 5), "kernel": kname,
                                  "frac_fp32_simt_nominal": round(tf / FP32_SIMT_NOMINAL_TFLOPS, 4),
                                  "parallelism": f"replicas x{world}", "gpu_launches": launches,
                                  "clocks": clk.summary(),
                                  "parity": {"rel_frobenius_max": max_over_ranks(rel, world),
                                             "tol": 1e-5 * math.sqrt(n), "reference": "fp64 product on the GPU"}}}


def _sharded_parity(Y, X, W_full, world, seed=11):
    """Full output Y [M, N] on this rank against an fp32 product: 64 complete
    rows and 64 complete columns (seeded, the same on every rank); then a
    checksum of all of Y gathered from every rank.  Collective."""
    import torch

    M, Nt = Y.shape
    g = torch.Generator().manual_seed(seed)
    rows = torch.randperm(M, generator=g)[:64].to(Y.device)
    cols = torch.randperm(Nt, generator=g)[:64].to(Y.device)
    r_rows = fp32_product(X[rows], W_full)
    r_cols = fp32_product(X, W_full[:, cols])
    err = max(max_rel(Y[rows], r_rows), max_rel(Y[:, cols], r_cols))
    sums = all_gather_floats(checksum(Y), world)
    return {"max_rel": max_over_ranks(err, world), "tol": LOWP_TOL,
            "ranks_identical": all(s == sums[0] for s in sums),
            "checked": "64 complete rows + 64 complete columns per rank vs fp32 product (TF32 off); "
                       "checksum of the full output all-gathered"}


def _sharded_gemm(cx, sharding, X, Wl, W_full, rank, world, steps, n_total, local_rank):
    """Column-sharded Y = X @ W with the full Y on every rank: the fused
    peer-store GEMM (graph-replayed, cross-GPU barriers inside) and, for
    comparison, GEMM + NCCL all-gather + gather kernel; each output checked
    on every rank after its timed region.  Returns (ms fused, ms nccl, kernel
    name, clocks, parity fused, parity nccl)."""
    import torch
    from cuop_b200 import peer

    M = X.size(0)
    pg = peer.PeerShardedGemm(Wl, rank, world, max_rows=M)
    clk = ClockSampler(local_rank)
    try:
        ms_peer, _ = time_graph(lambda i: pg.forward(X), steps, 3, world, align=lambda: peer.peer_barrier(pg.signals),
                                clock=clk)
        Y = pg.forward(X)
        kname = pg.last_kernel
        torch.cuda.synchronize()
        par_peer = _sharded_parity(Y, X, W_full, world)
        del Y
    finally:
        torch.cuda.synchronize()
        pg.close()
    sg = sharding.ColumnShardedGemm(Wl, world)
    Y = torch.empty(M, n_total, device=X.device, dtype=X.dtype)
    ms_nccl = time_loop(lambda i: sg.forward(X, out=Y), steps, 3, world)
    par_nccl = _sharded_parity(Y, X, W_full, world)
    del Y
    return ms_peer, ms_nccl, kname, clk.summary(), par_peer, par_nccl


def _config_gemm_lowp(cx, sharding, dev, steps, rank, world, local_rank, M, K, N_, dtype, x_scale, w_scale,
                      bf16_peak, seed):
    """One 16-bit GEMM config: single GPU, or column-sharded over the ranks
    with the full output on every rank.  X and W are generated from the same
    seed on every rank (each rank keeps its column block of W)."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    X = (torch.randn(M, K, device=dev, generator=g) * x_scale).to(dtype)
    W_full = (torch.randn(K, N_, device=dev, generator=g) * w_scale).to(dtype)
    nl = N_ // world
    Wl = W_full[:, rank * nl:(rank + 1) * nl].contiguous()
    Yl = torch.empty(M, nl, device=dev, dtype=dtype)
    clk_local = ClockSampler(local_rank)
    ms_local, launches = time_graph(lambda i: cx.gemm(X, Wl, Yl), steps, 3, world, clock=clk_local)
    kname = cx.last_kernel()
    res = {}
    if world == 1:
        ms = ms_local
        clocks = clk_local.summary()
        parity = _sharded_parity(Yl, X, W_full, 1)
    else:
        ms, ms_nccl, kname, clocks, parity, par_nccl = _sharded_gemm(cx, sharding, X, Wl, W_full, rank, world, steps,
                                                                     N_, local_rank)
        res["nccl_allgather_path"] = {"ms": round(ms_nccl, 4),
                                      "tflops_total": round(2 * M * K * N_ / (ms_nccl * 1e-3) / 1e12, 1),
                                      "parity": par_nccl}
    del Yl
    tf_local = 2 * M * K * nl / (ms_local * 1e-3) / 1e12
    out = {
        "tflops_total": round(2 * M * K * N_ / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4), "kernel": kname,
        "gemm_only_tflops_per_gpu": round(tf_local, 1), "frac_gemm_only": round(tf_local / bf16_peak, 4),
        "frac_spec_gemm_only": round(tf_local / SPEC_DENSE_16BIT_TFLOPS, 4),
        "parallelism": "single GPU" if world == 1 else
        f"W column-sharded x{world}; GEMM epilogue stores every tile into all ranks' outputs over NVLink",
        "clocks": clocks, "clocks_gemm_only": clk_local.summary(), "parity": parity, "gpu_launches_gemm_only": launches,
        **res}
    del X, W_full, Wl
    torch.cuda.empty_cache()
    return out


def _config_c3(cx, sharding, dev, steps, rank, world, local_rank, bf16_peak, peak_src):
    """fp16 GEMM 8192^3, A,B ~ N(0,1)/sqrt(K); N-sharded with the full C on every rank when world > 1."""
    n = 8192
    import torch

    out = _config_gemm_lowp(cx, sharding, dev, steps, rank, world, local_rank, n, n, n, torch.float16,
                            1 / math.sqrt(n), 1 / math.sqrt(n), bf16_peak, seed=301)
    out["peak_tflops"] = bf16_peak
    out["peak_source"] = f"{peak_src} bf16_tflops (burst)"
    return {"c3_fp16_gemm_8192": out}


def _config_c5(cx, sharding, dev, steps, rank, world, local_rank, bf16_peak):
    """bf16 linear 4096 x 8192 x 28672, X ~ N(0,1), W ~ N(0, 0.02); W column-sharded, full Y on every rank."""
    import torch

    out = _config_gemm_lowp(cx, sharding, dev, steps, rank, world, local_rank, 4096, 8192, 28672, torch.bfloat16,
                            1.0, 0.02, bf16_peak, seed=501)
    return {"c5_bf16_linear_4096x8192x28672": out}


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """CPU restatement of the reference's batched GEMM arithmetic (the
    reference has no CPU implementation) on all host threads; each step is a
    bounded batch sample of the C4 workload, sized so that the run ends in
    about a minute."""
    if rank != 0:
        return None
    import oracle as O

    nt = O.threads()
    A = O.to_lowp(O.normal((BATCH, BM, BK), seed=4), O.BF16)
    B = O.to_lowp(O.normal((BATCH, BK, BN), seed=5), O.BF16)
    t0 = time.perf_counter()
    O.gemm_batched_lowp(O.BF16, A, B, nthreads=nt)
    t_full = time.perf_counter() - t0
    budget = 60.0
    frac = min(1.0, budget / max(1e-9, (args.steps + args.warmup) * t_full))
    nb = max(64, int(BATCH * frac) // 64 * 64)
    As, Bs = A[:nb], B[:nb]
    for _ in range(args.warmup):
        O.gemm_batched_lowp(O.BF16, As, Bs, nthreads=nt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.gemm_batched_lowp(O.BF16, As, Bs, nthreads=nt)
    el = time.perf_counter() - t0
    gbs = args.steps * nb * C4_BYTES_PER_BATCH / el / 1e9
    sample = (f"each step: {nb} of the 4096 batches (128x128x64 bf16, fp32 accumulate) of the seeded workload; "
              f"oracle/cpu_ref.c, OpenMP {nt} threads")
    return {
        "impl": "reference", "metric": "bf16 batched GEMM 4096 x (128x128x64), batch-sharded: HBM GB/s",
        "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "bf16 strided-batched GEMM C[b] = A[b] B[b], batch 4096, M=N=128, K=64, "
                               "A,B ~ N(0,1), fp32 accumulate, bf16 out", "global_batch": BATCH,
                   "parallelism": "host CPU (rank 0)"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nt, "kind": "port", "sample": sample,
                         "cpu_model": cpu_model()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-configs", action="store_true", help="skip the other configs")
    ap.add_argument("--configs", default="c2,c1,c3,c5",
                    help="comma-separated subset of the other configs to run (c2, c1, c3, c5)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local_rank = env_rank()

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch

    torch.cuda.set_device(local_rank)
    dist_init(world)
    line = run_c4(args, rank, world, local_rank)
    if not args.no_configs:
        line["configs"] = run_configs(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_c4_baseline()
        if "configs" in line:
            cbs = cpu_config_baselines()
            if "c2_fp32_gemv_8192" in line["configs"]:
                cbs["c2_fp32_gemv_8192"] = cpu_gemv_baseline()
            for key, cb in cbs.items():
                if key in line["configs"]:
                    line["configs"][key]["cpu_baseline"] = cb
    elif rank == 0:
        line["cpu_baseline"] = None
    barrier(world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
