"""GEMM variant tuning: the offline sweep that writes the selection table, and
helpers to load / clear / override it (C ABI cuopx_tuning_*,
cuopx_set_gemm_variant).

    python -m cuop_b200.tuning --out cuop_b200/tuning_b200.txt

times the built-in choice and every applicable variant on a grid of
problem sizes (CUDA events over a CUDA graph of back-to-back launches,
inputs resident) and writes a rule, covering sizes within a factor sqrt(2)
of the measured point, wherever a variant beats the built-in choice by more
than 5 %, with the measured times in a comment.  `cuop_b200` loads
`tuning_b200.txt` when the library is first opened; the C++ facade loads a
table with cuopx_tuning_load_file.
"""
from __future__ import annotations

import argparse
import itertools
from pathlib import Path
from typing import Iterable, Optional

from . import _native as N

DEFAULT_TABLE = Path(__file__).resolve().parent / "tuning_b200.txt"

_DT_NAME = {N.F32: "f32", N.F64: "f64", N.F16: "f16", N.BF16: "bf16"}

# Candidate variants per element type (the table may name any of them).
CANDIDATES = {
    N.F16: ["tc2", "tc2_256x512", "tc_128x256", "tc_128x128"],
    N.BF16: ["tc2", "tc2_256x512", "tc_128x256", "tc_128x128"],
    N.F32: ["tf32x3_128x64", "tf32x3_128x128", "ffma"],
}

# Sweep grid: problems at powers of two; a rule covers the sizes within a
# factor sqrt(2) of its measured point, and is written only where a variant
# beats the built-in choice by more than MARGIN (the built-in thresholds stay
# in charge everywhere else).
MN_POINTS = [256, 512, 1024, 2048, 4096, 8192]
K_POINTS = [256, 1024, 4096, 8192]
BATCHED_POINTS = [(64, 64, 64), (128, 128, 64), (128, 128, 128), (256, 256, 64), (256, 256, 256), (512, 512, 128)]
MARGIN = 0.05


def variant_names() -> list[str]:
    out, i = [], 0
    while True:
        name = N.lib().cuopx_gemm_variant_name(i)
        if name is None:
            return out
        out.append(name.decode())
        i += 1


def load(path: Optional[Path] = None) -> int:
    """Load a table file (default: the shipped one); returns its row count."""
    p = Path(path) if path is not None else DEFAULT_TABLE
    N.check(N.lib().cuopx_tuning_load_file(str(p).encode()), f"cuopx_tuning_load_file({p})")
    return N.lib().cuopx_tuning_rows()


def load_text(text: str) -> int:
    N.check(N.lib().cuopx_tuning_load(text.encode()), "cuopx_tuning_load")
    return N.lib().cuopx_tuning_rows()


def clear() -> None:
    N.check(N.lib().cuopx_tuning_clear(), "cuopx_tuning_clear")


def force(variant: Optional[str]) -> None:
    """Force one variant process-wide (None / "auto" restores the selection)."""
    N.check(N.lib().cuopx_set_gemm_variant(None if variant is None else variant.encode()),
            f"cuopx_set_gemm_variant({variant})")


def _around(p: int) -> str:
    """Inclusive range of sizes within a factor sqrt(2) of p."""
    return f"{int(p * 0.7072) + 1}:{int(p * 1.4142)}"


def time_variant(variant: str, A, B, C, batch: int, launches: int = 10) -> Optional[float]:
    """Median ms per launch of `variant` ("auto": the built-in choice; None
    when the variant cannot run the problem)."""
    import torch
    from . import ops

    def run():
        if batch > 1:
            ops.batched_gemm(A, B, C)
        else:
            ops.gemm(A, B, C)

    force(None if variant == "auto" else variant)
    try:
        run()
        torch.cuda.synchronize()
        got = ops.last_kernel()
        if variant != "auto" and not _kernel_matches(variant, got):
            return None  # declined: the built-in choice ran instead
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(launches):
                run()
        # Warm-up of at least ~20 ms of device work, so that the clock has
        # settled before the timed replays whatever ran before.
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        one = max(e0.elapsed_time(e1), 1e-3)
        for _ in range(min(200, int(20.0 / one))):
            g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / launches)
        return sorted(ts)[1]
    finally:
        force(None)


def _kernel_matches(variant: str, kernel: str) -> bool:
    expect = {"tc2": "gemm_tc2_256x256", "tc2_256x512": "gemm_tc2_256x512", "tc_128x256": "gemm_tc_128x256", "tc_128x128": "gemm_tc_128x128",
              "tf32x3_128x64": "gemm_tf32x3_128x64", "tf32x3_128x128": "gemm_tf32x3_128x128",
              "ffma": "gemm_f32_", "generic": "gemm_simt_generic"}[variant]
    return kernel.startswith(expect)


def sweep(dtypes: Iterable[int] = (N.F16, N.BF16, N.F32), cap: int = 8192, log=print) -> list[str]:
    """Time the built-in choice and every candidate on the sweep grid; returns
    table lines (rules only where a candidate wins by more than MARGIN)."""
    import torch
    from . import ops

    dev = torch.device("cuda", torch.cuda.current_device())
    tdt = {N.F16: torch.float16, N.BF16: torch.bfloat16, N.F32: torch.float32}
    lines = ["# dtype transA transB M N K batch variant   (measured point: built-in time vs winner, ms per launch)"]
    clear()
    shapes = [(m, n, k, 1) for m, n, k in itertools.product(MN_POINTS, MN_POINTS, K_POINTS)
              if max(m, n, k) <= cap]
    shapes += [(m, n, k, max(2, (64 << 20) // (m * n * 2))) for m, n, k in BATCHED_POINTS]
    for dt in dtypes:
        for M, Nn, K, batch in shapes:
            shape_a = (batch, M, K) if batch > 1 else (M, K)
            A = torch.randn(*shape_a, device=dev).to(tdt[dt])
            B = torch.randn(*((batch, K, Nn) if batch > 1 else (K, Nn)), device=dev).to(tdt[dt])
            C = torch.empty(*((batch, M, Nn) if batch > 1 else (M, Nn)), device=dev, dtype=tdt[dt])
            t_auto = time_variant("auto", A, B, C, batch)
            auto_kernel = ops.last_kernel()
            times = {v: t for v in CANDIDATES[dt] if (t := time_variant(v, A, B, C, batch)) is not None}
            # The built-in choice again after the candidates: the better of
            # its two times, so a clock change across the candidates does
            # not turn into a rule.
            t_auto = min(t_auto, time_variant("auto", A, B, C, batch))
            del A, B, C
            if not times:
                continue
            best = min(times, key=times.get)
            desc = f"{M}x{Nn}x{K} batch {batch}: built-in {t_auto:.4f} ({auto_kernel}), {best} {times[best]:.4f}"
            if times[best] < (1.0 - MARGIN) * t_auto and not _kernel_matches(best, auto_kernel):
                bat = "1:1" if batch == 1 else "2:"
                lines.append(f"{_DT_NAME[dt]} 0 0 {_around(M)} {_around(Nn)} {_around(K)} {bat} {best}   # {desc}")
                log(lines[-1])
            else:
                log(f"# keep built-in  {_DT_NAME[dt]} {desc}")
    return lines


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default=str(DEFAULT_TABLE))
    ap.add_argument("--cap", type=int, default=8192, help="largest representative size")
    args = ap.parse_args(argv)
    lines = sweep(cap=args.cap)
    Path(args.out).write_text("\n".join(lines) + "\n")
    print(f"wrote {len(lines) - 1} rows to {args.out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
