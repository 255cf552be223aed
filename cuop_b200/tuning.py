"""GEMM variant tuning: the offline sweep that writes the selection table, and
helpers to load / clear / override it (C ABI cuopx_tuning_*,
cuopx_set_gemm_variant).

    python -m cuop_b200.tuning --out cuop_b200/tuning_b200.txt

times every applicable variant on one representative problem per size
bucket (CUDA events over a CUDA graph of back-to-back launches, inputs
resident) and writes one table row per bucket naming the fastest variant,
with the measured times in a comment.  `cuop_b200` loads
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
    N.F16: ["tc2", "tc_128x256", "tc_128x128"],
    N.BF16: ["tc2", "tc_128x256", "tc_128x128"],
    N.F32: ["tf32x3_128x64", "tf32x3_128x128", "ffma"],
}

# Size buckets: (lo, hi) inclusive, hi None = unbounded; the representative
# size is hi/2 (4x lo, capped, for the open bucket).
MN_BUCKETS = [(1, 512), (513, 2048), (2049, None)]
K_BUCKETS = [(1, 1024), (1025, None)]
BATCH_BUCKETS = [(1, 1), (2, None)]


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


def _rep(lo: int, hi: Optional[int], cap: int) -> int:
    if hi is None:
        return min(cap, 4 * lo) // 64 * 64 or 64
    return max(64, hi // 2 // 64 * 64)


def _fmt_range(lo: int, hi: Optional[int]) -> str:
    return f"{lo}:{'' if hi is None else hi}"


def time_variant(variant: str, A, B, C, batch: int, launches: int = 10) -> Optional[float]:
    """Median ms per launch of `variant` (None when it cannot run the problem)."""
    import torch
    from . import ops

    def run():
        if batch > 1:
            ops.batched_gemm(A, B, C)
        else:
            ops.gemm(A, B, C)

    force(variant)
    try:
        run()
        torch.cuda.synchronize()
        got = ops.last_kernel()
        if not _kernel_matches(variant, got):
            return None  # declined: the built-in choice ran instead
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(launches):
                run()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    expect = {"tc2": "gemm_tc2_", "tc_128x256": "gemm_tc_128x256", "tc_128x128": "gemm_tc_128x128",
              "tf32x3_128x64": "gemm_tf32x3_128x64", "tf32x3_128x128": "gemm_tf32x3_128x128",
              "ffma": "gemm_f32_", "generic": "gemm_simt_generic"}[variant]
    return kernel.startswith(expect)


def sweep(dtypes: Iterable[int] = (N.F16, N.BF16, N.F32), cap: int = 8192, log=print) -> list[str]:
    """Time the candidates on one problem per bucket; returns table lines."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device())
    tdt = {N.F16: torch.float16, N.BF16: torch.bfloat16, N.F32: torch.float32}
    lines = ["# dtype transA transB M N K batch variant   (fastest measured; times in ms per launch)"]
    clear()
    for dt in dtypes:
        for (mlo, mhi), (nlo, nhi), (klo, khi), (blo, bhi) in itertools.product(MN_BUCKETS, MN_BUCKETS, K_BUCKETS,
                                                                                BATCH_BUCKETS):
            M, Nn, K = _rep(mlo, mhi, cap), _rep(nlo, nhi, cap), _rep(klo, khi, cap)
            batch = 1 if bhi == 1 else max(2, min(256, (64 << 20) // max(1, M * Nn * 2)))
            if batch > 1 and M * Nn * K > (1 << 30):
                continue  # large batched problems behave like the non-batched bucket
            shape = (batch, M, K) if batch > 1 else (M, K)
            A = torch.randn(*shape, device=dev).to(tdt[dt])
            B = torch.randn(*((batch, K, Nn) if batch > 1 else (K, Nn)), device=dev).to(tdt[dt])
            C = torch.empty(*((batch, M, Nn) if batch > 1 else (M, Nn)), device=dev, dtype=tdt[dt])
            times = {}
            for v in CANDIDATES[dt]:
                t = time_variant(v, A, B, C, batch)
                if t is not None:
                    times[v] = t
            del A, B, C
            if not times:
                continue
            best = min(times, key=times.get)
            row = (f"{_DT_NAME[dt]} 0 0 {_fmt_range(mlo, mhi)} {_fmt_range(nlo, nhi)} {_fmt_range(klo, khi)} "
                   f"{_fmt_range(blo, bhi)} {best}")
            note = ", ".join(f"{k} {v:.4f}" for k, v in sorted(times.items(), key=lambda kv: kv[1]))
            lines.append(f"{row}   # {M}x{Nn}x{K} batch {batch}: {note}")
            log(lines[-1])
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
