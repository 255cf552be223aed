#!/usr/bin/env python
"""Benchmark of the cuop_b200 dense BLAS hot path on B200.

Headline workload (one JSON line, rank 0): fp32 GEMV, y = 1.0*A*x + 0.0*y with
A 8192 x 8192 row-major, plus the transposed (A^T x) variant; A, x uniform
[-1, 1).  One step = one plain + one transposed GEMV on a fresh input set
(4 sets of 256 MiB rotated, so every A read comes from HBM, not the 126 MB
L2).  Metric: HBM GB/s of algorithmic traffic (A once, x once, y written once
per GEMV).  The GEMV path does not shard, so `--gpus N` runs N replicas.

The same line carries, under "configs", the other GEMM shapes of the path:
fp32 GEMM 1024^3, fp16 GEMM 8192^3, bf16 batched 4096 x 128x128x64
(batch-sharded, no collective), bf16 linear 4096 x 8192 x 28672.  At N>1 the
two large GEMMs are column-sharded and the full output is assembled on every
rank by the GEMM epilogue's own stores into the peers' outputs over NVLink
(GEMM + NCCL all-gather + gather kernel is timed beside it).
`--configs c3` (etc.) runs a subset of them.

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

GEMV_N = 8192
GEMV_BYTES = (GEMV_N * GEMV_N + 2 * GEMV_N) * 4  # A + x + y (beta = 0: y not read)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FP32_SIMT_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# Nominal B200 figures, reported beside the measured-peak fractions.
SPEC_HBM_GBS = 8000.0
SPEC_DENSE_16BIT_TFLOPS = 2250.0

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one
# ncu capture of the two fp32 GEMV kernels at 8192 x 8192.
NCU_TRAFFIC_BYTES = {"gemv_t_lsu": 272088832, "gemv_n_xreg": 272280576}


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


def time_graph(fn, steps, warmup, world, align=None):
    """Device time (ms per call) of `steps` calls of fn replayed as one CUDA
    graph after `warmup` eager calls; max over ranks.  `align`, if given, is
    launched on the stream just before the timed replay (a cross-GPU barrier,
    so that host-side skew between ranks stays out of the timed region)."""
    import torch

    for i in range(warmup):
        fn(i)
    g, _ = capture_graph(fn, steps)
    g.replay()  # first replay uploads the graph
    barrier(world)
    if align is not None:
        align()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    g.replay()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    barrier(world)
    del g
    return max_over_ranks(ms, world)


def time_loop(fn, steps, warmup, world, stream=None):
    """Eager device time (ms per call) of `steps` calls, max over ranks (used
    where a step holds NCCL collectives, which stay out of graphs)."""
    import torch

    for _ in range(warmup):
        fn(0)
    barrier(world)
    s = stream or torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        fn(i)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    barrier(world)
    return max_over_ranks(ms, world)


# --------------------------------------------------------------------------- GEMV (headline)
def gemv_inputs(dev, sets: int, seed: int = 0):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    An = [torch.rand(GEMV_N, GEMV_N, device=dev, generator=g).mul_(2).sub_(1) for _ in range(sets)]
    At = [torch.rand(GEMV_N, GEMV_N, device=dev, generator=g).mul_(2).sub_(1) for _ in range(sets)]
    x = torch.rand(GEMV_N, device=dev, generator=g).mul_(2).sub_(1)
    return An, At, x


def run_gemv(args, rank, world, local_rank):
    import torch
    import cuop_b200 as cx

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    sets = 2
    An, At, x = gemv_inputs(dev, sets, seed=1234 + rank)
    yn = torch.empty(GEMV_N, device=dev)
    yt = torch.empty(GEMV_N, device=dev)
    stream = torch.cuda.current_stream()

    def step(i):
        cx.gemv(An[i % sets], x, yn)
        cx.gemv(At[i % sets], x, yt, trans=True)

    for i in range(args.warmup):
        step(i)
    barrier(world)

    K = args.steps
    # The timed region replays one CUDA graph of K steps (2K kernels).
    g_step, launches = capture_graph(step, K)
    kn = kt = None
    cx.gemv(An[0], x, yn)
    kn = cx.last_kernel()
    cx.gemv(At[0], x, yt, trans=True)
    kt = cx.last_kernel()
    g_step.replay()
    barrier(world)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e_start.record(stream)
        g_step.replay()
        e_end.record(stream)
        torch.cuda.synchronize()
    ms_local = e_start.elapsed_time(e_end) / K
    del g_step
    barrier(world)
    ms = max_over_ranks(ms_local, world)
    # Per-kernel device time: each kernel alone, back to back, same rotation.
    t_n = time_graph(lambda i: cx.gemv(An[i % sets], x, yn), K, 2, world)
    t_t = time_graph(lambda i: cx.gemv(At[i % sets], x, yt, trans=True), K, 2, world)

    hbm, bf16, bf16_sus, peak_src = load_peaks()
    value = world * 2 * GEMV_BYTES / (ms * 1e-3) / 1e9
    dom_name, dom_ms = (kt, t_t) if t_t >= t_n else (kn, t_n)
    achieved = GEMV_BYTES / (dom_ms * 1e-3) / 1e9
    kernels = {
        kn: {"ms": round(t_n, 5), "gbs": round(GEMV_BYTES / (t_n * 1e-3) / 1e9, 1),
             "frac": round(GEMV_BYTES / (t_n * 1e-3) / 1e9 / hbm, 4)},
        kt: {"ms": round(t_t, 5), "gbs": round(GEMV_BYTES / (t_t * 1e-3) / 1e9, 1),
             "frac": round(GEMV_BYTES / (t_t * 1e-3) / 1e9 / hbm, 4)},
    }

    e2e = gemv_e2e_plugin(args, rank, world, local_rank, An, At)
    e2e_operator = gemv_e2e(args, rank, world, local_rank, An[0], At[0], x)
    line = {
        "metric": "GEMV fp32 8192x8192 (plain + transposed) HBM GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "fp32 GEMV y=1.0*A*x+0.0*y, M=N=8192 row-major, plain + transposed (A^T x), "
                               "A,x ~ U[-1,1)", "parallelism": f"replicas x{world} (GEMV does not shard)",
                   "l2": "inputs larger than L2: 4 x 256 MiB matrices rotated per step",
                   "bytes_per_step": 2 * GEMV_BYTES},
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": round(achieved, 1), "peak": hbm,
                     "peak_source": f"{peak_src} hbm_gbs (burst copy)", "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "frac_spec": round(achieved / SPEC_HBM_GBS, 4),
                     "spec_peak": SPEC_HBM_GBS, "traffic": NCU_TRAFFIC_BYTES.get(dom_name),
                     "algorithmic_bytes": GEMV_BYTES},
        "kernels": kernels,
        "gpu_launches": launches,
        "timing": "timed region = one CUDA graph replay of K steps; per-kernel times from graphs of K launches",
        "clocks": clk.summary(),
        "e2e": e2e,
        "e2e_operator_path": e2e_operator,
    }
    return line


def gemv_e2e_plugin(args, rank, world, local_rank, An, At):
    """Same metric through the public API in the plugin's usage model
    (GemvJITPlugin: the matrix is the plugin's weight, set once and resident;
    each Execute takes x and returns y): every step brings a fresh x from
    pinned host memory to the device, runs both GEMVs on the step's resident
    matrices, puts both results in pinned host memory and waits for them on
    the host.  x is staged by the library's copy kernel reading the pinned
    buffer (cuopx_copy) and the GEMVs write y straight into pinned host
    memory, so the step is three kernels with no copy-engine transfer."""
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

    # One CUDA graph per rotation slot holds the step's three launches (host
    # launch cost of one replay instead of three API calls).
    graphs = []
    for k in range(sets):
        body(k)
        torch.cuda.synchronize()
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gk):
            body(k)
        graphs.append(gk)

    # The host copy of the results is the device's answer.
    yn = torch.empty(GEMV_N, device=dev)
    yt = torch.empty(GEMV_N, device=dev)
    graphs[0].replay()
    stream.synchronize()
    cx.gemv(An[0], dx, yn)
    cx.gemv(At[0], dx, yt, trans=True)
    torch.cuda.synchronize()
    if not (torch.equal(hy[0], yn.cpu()) and torch.equal(hy[1], yt.cpu())):
        raise RuntimeError("GEMV results in pinned host memory differ from the device results")

    def step(i):
        graphs[i % sets].replay()
        stream.synchronize()  # the host has the step's results

    steps = max(5, min(args.steps, 200))
    ms = time_loop(step, steps, 3, world)
    del graphs
    return {"value": round(world * 2 * GEMV_BYTES / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": GEMV_N * 4, "d2h_bytes_per_step": 2 * GEMV_N * 4,
            "ms_per_step": round(ms, 4), "steps": steps,
            "path": "cuop_b200.copy + cuop_b200.gemv (C ABI) with the matrices resident as plugin weights; per "
                    "step x read from pinned host memory by the copy kernel, both GEMVs writing y into pinned host "
                    "memory, replayed as one CUDA graph, then host synchronisation"}


def gemv_e2e(args, rank, world, local_rank, An, At, x):
    """Same metric through the public API with pinned host buffers: H2D of
    both matrices and x, both GEMVs, D2H of both results, every step."""
    import torch
    import cuop_b200 as cx

    dev = torch.device("cuda", local_rank)
    hA = An.cpu().pin_memory()
    hAt = At.cpu().pin_memory()
    hx = x.cpu().pin_memory()
    hyn = torch.empty(GEMV_N, pin_memory=True)
    hyt = torch.empty(GEMV_N, pin_memory=True)
    dA = torch.empty_like(An)
    dAt = torch.empty_like(At)
    dx = torch.empty_like(x)
    yn = torch.empty(GEMV_N, device=dev)
    yt = torch.empty(GEMV_N, device=dev)

    def step(_):  # the operator API's model: the matrix itself is the per-call input
        dA.copy_(hA, non_blocking=True)
        dAt.copy_(hAt, non_blocking=True)
        dx.copy_(hx, non_blocking=True)
        cx.gemv(dA, dx, yn)
        cx.gemv(dAt, dx, yt, trans=True)
        hyn.copy_(yn, non_blocking=True)
        hyt.copy_(yt, non_blocking=True)

    steps = max(3, min(args.steps, 10))
    ms = time_loop(step, steps, 2, world)
    return {"value": round(world * 2 * GEMV_BYTES / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": 2 * GEMV_N * GEMV_N * 4 + GEMV_N * 4, "d2h_bytes_per_step": 2 * GEMV_N * 4,
            "ms_per_step": round(ms, 4), "steps": steps,
            "path": "Gemv<T>::Forward model: both 256 MiB matrices H2D every step (PCIe-bound)"}


# --------------------------------------------------------------------------- CPU baseline (oracle)
def cpu_gemv_baseline(budget_s: float = 4.0):
    """The CPU restatement of the reference GEMV on all host threads, full
    8192^2 plain + transposed, repeated for about `budget_s` seconds."""
    import numpy as np
    import oracle as O

    nt = O.threads()
    A = O.uniform((GEMV_N, GEMV_N), seed=0)
    x = O.uniform(GEMV_N, seed=1)
    O.gemv_f32(A, x, nthreads=nt)  # warm-up (page-in)
    reps, t0 = 0, time.perf_counter()
    while True:
        O.gemv_f32(A, x, nthreads=nt)
        O.gemv_f32(A, x, trans=True, nthreads=nt)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    gbs = reps * 2 * GEMV_BYTES / el / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"full workload: {reps} x (plain + transposed) fp32 GEMV 8192^2 in {el:.2f} s, "
                      f"oracle/cpu_ref.c, OpenMP {nt} threads"}


def cpu_config_baselines(budget_s: float = 1.5) -> dict:
    """The oracle (CPU restatement of the reference kernels' arithmetic) on
    the GEMM configs, all host threads: C1 and C4 in full, C3 and C5 on a
    64-row slab of A with the full-problem time extrapolated by rows."""
    import numpy as np
    import oracle as O

    nt = O.threads()

    def timed(fn):
        fn()  # page-in
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s or reps >= 20:
                return el / reps

    out = {}
    n = 1024
    A, B = O.uniform((n, n), seed=0), O.uniform((n, n), seed=1)
    t = timed(lambda: O.gemm_f32(A, B, nthreads=nt))
    out["c1_fp32_gemm_1024"] = {"value": round(2 * n ** 3 / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt,
                                "kind": "port", "sample": f"full 1024^3 fp32 GEMM, {t * 1e3:.1f} ms"}
    n, rows = 8192, 64
    A = O.to_lowp(O.normal((rows, n), seed=2) / math.sqrt(n), O.F16)
    B = O.to_lowp(O.normal((n, n), seed=3) / math.sqrt(n), O.F16)
    t = timed(lambda: O.gemm_lowp(O.F16, A, B, nthreads=nt))
    out["c3_fp16_gemm_8192"] = {"value": round(2 * rows * n * n / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt,
                                "kind": "port", "sample": f"64-row slab of the 8192^3 fp16 GEMM, {t * 1e3:.0f} ms; "
                                                          f"extrapolated full problem {t * n / rows:.1f} s"}
    bt, M, N_, K = 4096, 128, 128, 64
    A = O.to_lowp(O.normal((bt, M, K), seed=4), O.BF16)
    B = O.to_lowp(O.normal((bt, K, N_), seed=5), O.BF16)
    t = timed(lambda: O.gemm_batched_lowp(O.BF16, A, B, nthreads=nt))
    out["c4_bf16_batched_4096x128x128x64"] = {
        "value": round(bt * (M * K + K * N_ + M * N_) * 2 / t / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
        "sample": f"full 4096 x 128x128x64 bf16 batched GEMM, {t * 1e3:.0f} ms"}
    M, K, N_ = 4096, 8192, 28672
    X = O.to_lowp(O.normal((rows, K), seed=6), O.BF16)
    W = O.to_lowp(O.normal((K, N_), seed=7) * 0.02, O.BF16)
    t = timed(lambda: O.gemm_lowp(O.BF16, X, W, nthreads=nt))
    out["c5_bf16_linear_4096x8192x28672"] = {
        "value": round(2 * rows * K * N_ / t / 1e12, 4), "unit": "TFLOP/s", "cores": nt, "kind": "port",
        "sample": f"64-row slab of the 4096 x 8192 x 28672 bf16 GEMM, {t * 1e3:.0f} ms; "
                  f"extrapolated full problem {t * M / rows:.1f} s"}
    return out


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
    # The memory-bound batched config runs before the tensor-bound GEMMs:
    # right after the 8192^3 GEMM at the power cap it read up to ~10 % lower
    # than the same kernel measured alone on the same part.
    if "c1" in want:
        out.update(_config_c1(cx, dev, g, steps, world))
    if "c4" in want:
        out.update(_config_c4(cx, sharding, dev, g, steps, rank, world, hbm))
    if "c3" in want:
        out.update(_config_c3(cx, sharding, dev, g, steps, rank, world, bf16_peak, peak_src))
    if "c5" in want:
        out.update(_config_c5(cx, sharding, dev, g, steps, rank, world, bf16_peak))
    return out


def _config_c1(cx, dev, g, steps, world):
    """fp32 GEMM 1024^3 (replicas)."""
    import torch

    n = 1024
    A = torch.rand(n, n, device=dev, generator=g) * 2 - 1
    B = torch.rand(n, n, device=dev, generator=g) * 2 - 1
    C = torch.empty(n, n, device=dev)
    ms = time_graph(lambda i: cx.gemm(A, B, C), steps * 4, 5, world)
    tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
    return {"c1_fp32_gemm_1024": {"tflops_total": round(world * tf, 3), "ms": round(ms, 5),
                                  "kernel": cx.last_kernel(),
                                  "frac_fp32_simt_nominal": round(tf / FP32_SIMT_NOMINAL_TFLOPS, 4),
                                  "parallelism": f"replicas x{world}"}}


def _sharded_gemm(cx, sharding, X, Wl, rank, world, steps, n_total):
    """Column-sharded Y = X @ W with the full Y on every rank: the fused
    peer-store GEMM (graph-replayed, cross-GPU barriers inside) and, for
    comparison, GEMM + NCCL all-gather + gather kernel.  Returns
    (ms fused, ms nccl, kernel name)."""
    import torch
    from cuop_b200 import peer

    M = X.size(0)
    pg = peer.PeerShardedGemm(Wl, rank, world, max_rows=M)
    try:
        ms_peer = time_graph(lambda i: pg.forward(X), steps, 3, world, align=lambda: peer.peer_barrier(pg.signals))
        pg.forward(X)
        kname = pg.last_kernel
    finally:
        torch.cuda.synchronize()
        pg.close()
    sg = sharding.ColumnShardedGemm(Wl, world)
    Y = torch.empty(M, n_total, device=X.device, dtype=X.dtype)
    ms_nccl = time_loop(lambda i: sg.forward(X, out=Y), steps, 3, world)
    del Y
    return ms_peer, ms_nccl, kname


def _config_c3(cx, sharding, dev, g, steps, rank, world, bf16_peak, peak_src):
    """fp16 GEMM 8192^3; N-sharded with an all-gather of C when world > 1."""
    import torch

    n = 8192
    A = (torch.randn(n, n, device=dev, generator=g) / math.sqrt(n)).half()
    Wfull_cols = n // world
    Wl = (torch.randn(n, Wfull_cols, device=dev, generator=g) / math.sqrt(n)).half()
    Cl = torch.empty(n, Wfull_cols, device=dev, dtype=torch.half)
    ms_local = time_graph(lambda i: cx.gemm(A, Wl, Cl), steps, 3, world)
    kname = cx.last_kernel()
    del Cl
    res = {}
    if world == 1:
        ms = ms_local
    else:
        ms, ms_nccl, kname = _sharded_gemm(cx, sharding, A, Wl, rank, world, steps, n)
        res["nccl_allgather_path"] = {"ms": round(ms_nccl, 4),
                                      "tflops_total": round(2 * n ** 3 / (ms_nccl * 1e-3) / 1e12, 1)}
    tf_local = 2 * n * n * Wfull_cols / (ms_local * 1e-3) / 1e12
    res = {
        "tflops_total": round(2 * n ** 3 / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4), "kernel": kname,
        "gemm_only_tflops_per_gpu": round(tf_local, 1), "frac_gemm_only": round(tf_local / bf16_peak, 4),
        "frac_spec_gemm_only": round(tf_local / SPEC_DENSE_16BIT_TFLOPS, 4), "peak_tflops": bf16_peak, "peak_source": f"{peak_src} bf16_tflops (burst)",
        "parallelism": "single GPU" if world == 1 else
        f"N-sharded x{world}; GEMM epilogue stores every tile into all ranks' outputs over NVLink", **res}
    del A, Wl
    torch.cuda.empty_cache()
    return {"c3_fp16_gemm_8192": res}


def _config_c4(cx, sharding, dev, g, steps, rank, world, hbm):
    """bf16 batched 4096 x (128x128x64), batch-sharded, no collective."""
    import torch

    batch, M, N_, K = 4096, 128, 128, 64
    b0, b1 = sharding.shard_range(batch, rank, world)
    lb = b1 - b0
    per_set = lb * (M * K + K * N_ + M * N_) * 2
    sets = max(2, math.ceil(400e6 / per_set))
    As = [torch.randn(lb, M, K, device=dev, generator=g).bfloat16() for _ in range(sets)]
    Bs = [torch.randn(lb, K, N_, device=dev, generator=g).bfloat16() for _ in range(sets)]
    Cs = [torch.empty(lb, M, N_, device=dev, dtype=torch.bfloat16) for _ in range(sets)]
    ms = time_graph(lambda i: cx.batched_gemm(As[i % sets], Bs[i % sets], Cs[i % sets]), steps * 4, 5, world)
    bytes_total = batch * (M * K + K * N_ + M * N_) * 2
    gbs_local = lb * (M * K + K * N_ + M * N_) * 2 / (ms * 1e-3) / 1e9
    res = {
        "gbs_total": round(bytes_total / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 5), "kernel": cx.last_kernel(),
        "tflops_total": round(2 * batch * M * N_ * K / (ms * 1e-3) / 1e12, 2),
        "frac_hbm_per_gpu": round(gbs_local / hbm, 4), "frac_spec_hbm_per_gpu": round(gbs_local / SPEC_HBM_GBS, 4),
        "l2": f"{sets} rotated input sets > L2",
        "parallelism": f"batch-sharded x{world}, no collective"}
    del As, Bs, Cs
    torch.cuda.empty_cache()
    return {"c4_bf16_batched_4096x128x128x64": res}


def _config_c5(cx, sharding, dev, g, steps, rank, world, bf16_peak):
    """bf16 linear 4096 x 8192 x 28672, W column-sharded, all-gather of Y."""
    import torch

    M, K, N_ = 4096, 8192, 28672
    X = torch.randn(M, K, device=dev, generator=g).bfloat16()
    nl = N_ // world
    Wl = (torch.randn(K, nl, device=dev, generator=g) * 0.02).bfloat16()
    Yl = torch.empty(M, nl, device=dev, dtype=torch.bfloat16)
    ms_local = time_graph(lambda i: cx.gemm(X, Wl, Yl), steps, 3, world)
    kname = cx.last_kernel()
    del Yl
    res = {}
    if world > 1:
        ms, ms_nccl, kname = _sharded_gemm(cx, sharding, X, Wl, rank, world, steps, N_)
        res["nccl_allgather_path"] = {"ms": round(ms_nccl, 4),
                                      "tflops_total": round(2 * M * K * N_ / (ms_nccl * 1e-3) / 1e12, 1)}
    else:
        ms = ms_local
    tf_local = 2 * M * K * nl / (ms_local * 1e-3) / 1e12
    res = {
        "tflops_total": round(2 * M * K * N_ / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4), "kernel": kname,
        "gemm_only_tflops_per_gpu": round(tf_local, 1), "frac_gemm_only": round(tf_local / bf16_peak, 4),
        "frac_spec_gemm_only": round(tf_local / SPEC_DENSE_16BIT_TFLOPS, 4),
        "parallelism": "single GPU" if world == 1 else
        f"W column-sharded x{world}; GEMM epilogue stores every tile of Y into all ranks' outputs over NVLink",
        **res}
    del X, Wl
    torch.cuda.empty_cache()
    return {"c5_bf16_linear_4096x8192x28672": res}


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """CPU restatement of the reference GEMV path (the reference has no CPU
    implementation) on all host threads; each step is a bounded row sample of
    the 8192^2 plain + transposed workload."""
    if rank != 0:
        return None
    import numpy as np
    import oracle as O

    nt = O.threads()
    A = O.uniform((GEMV_N, GEMV_N), seed=0)
    x = O.uniform(GEMV_N, seed=1)
    t0 = time.perf_counter()
    O.gemv_f32(A, x, nthreads=nt)
    O.gemv_f32(A, x, trans=True, nthreads=nt)
    t_full = time.perf_counter() - t0
    budget = 90.0
    frac = min(1.0, budget / max(1e-9, (args.steps + args.warmup) * t_full))
    rows = max(64, int(GEMV_N * frac) // 64 * 64)
    As = np.ascontiguousarray(A[:rows])
    xs_t = np.ascontiguousarray(x[:rows])
    sample_bytes = (rows * GEMV_N + GEMV_N + rows) * 4 + (rows * GEMV_N + rows + GEMV_N) * 4

    def step():
        O.gemv_f32(As, x, nthreads=nt)          # rows x 8192 plain
        O.gemv_f32(As, xs_t, trans=True, nthreads=nt)  # sum over `rows` rows, 8192 outputs

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gbs = args.steps * sample_bytes / el / 1e9
    sample = (f"each step: plain GEMV on a {rows}x8192 row slab + transposed GEMV over the same {rows} rows "
              f"(8192 outputs) of the seeded 8192^2 fp32 workload; oracle/cpu_ref.c, OpenMP {nt} threads")
    return {
        "impl": "reference", "metric": "GEMV fp32 8192x8192 (plain + transposed) HBM GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "fp32 GEMV y=1.0*A*x+0.0*y, M=N=8192 row-major, plain + transposed (A^T x), "
                               "A,x ~ U[-1,1)", "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nt, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-configs", action="store_true", help="skip the other GEMM configs")
    ap.add_argument("--configs", default="c1,c3,c4,c5",
                    help="comma-separated subset of the other configs to run (c1, c3, c4, c5)")
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
    line = run_gemv(args, rank, world, local_rank)
    if not args.no_configs:
        line["configs"] = run_configs(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_gemv_baseline()
        if "configs" in line:
            for key, cb in cpu_config_baselines().items():
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
