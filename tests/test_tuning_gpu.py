"""GEMM variant selection through the tuning table (cuopx_tuning_*) and the
process-wide override: the named variant runs, unsupported rows fall back to
the built-in choice, the fp32 mode wins over the table, and results stay
within tolerance of the oracle whichever variant runs."""
import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from cuop_b200 import _native as N
from cuop_b200 import tuning
from helpers import lowp_bits, to_dev_f32, to_dev_lowp

pytestmark = pytest.mark.gpu


@pytest.fixture
def table():
    yield tuning.load_text
    tuning.clear()
    tuning.force(None)


def test_table_routes_each_bucket(dev, table):
    table("""
bf16 0 0 1:1024 1:1024 * 1:1 tc_128x256     # small: wide 1-SM tile
bf16 0 0 1025: * * 1:1 tc_128x128
bf16 0 0 * * * 2: tc2                        # batched through the pair kernel
f32  0 0 * * * * tf32x3_128x128
""")
    A = torch.randn(512, 256, device=dev).bfloat16()
    B = torch.randn(256, 768, device=dev).bfloat16()
    C = cx.gemm(A, B)
    assert cx.last_kernel() == "gemm_tc_128x256"
    ref = A.float() @ B.float()
    assert O.max_relative(C.float().cpu().numpy(), ref.cpu().numpy()) <= 1e-2
    A = torch.randn(2048, 256, device=dev).bfloat16()
    cx.gemm(A, B)
    assert cx.last_kernel() == "gemm_tc_128x128"
    Ab = torch.randn(8, 256, 128, device=dev).bfloat16()
    Bb = torch.randn(8, 128, 512, device=dev).bfloat16()
    Cb = cx.batched_gemm(Ab, Bb)
    assert cx.last_kernel() == "gemm_tc2_256x256"
    refb = torch.bmm(Ab.float(), Bb.float())
    assert O.max_relative(Cb.float().cpu().numpy(), refb.cpu().numpy()) <= 1e-2
    A32 = O.uniform((300, 400), seed=1)
    B32 = O.uniform((400, 200), seed=2)
    C32 = cx.gemm(to_dev_f32(A32, dev), to_dev_f32(B32, dev))
    assert cx.last_kernel() == "gemm_tf32x3_128x128"
    exact = A32.astype(np.float64) @ B32.astype(np.float64)
    assert O.rel_frobenius(C32.cpu().numpy(), exact) <= 1e-5 * np.sqrt(400)


def test_unsupported_row_falls_back(dev, table):
    table("f32 * * * * * * tc2\nbf16 * * * * * * tf32x3_128x64\n")
    A = torch.randn(256, 256, device=dev)
    cx.gemm(A, A.clone())
    assert cx.last_kernel().startswith("gemm_tf32x3_")  # built-in choice for fp32
    X = torch.randn(256, 256, device=dev).bfloat16()
    cx.gemm(X, X.clone())
    assert cx.last_kernel().startswith("gemm_tc")


def test_fp32_mode_wins_over_table(dev, table, fp32_ffma):
    table("f32 * * * * * * tf32x3_128x64\n")
    A32 = O.uniform((256, 256), seed=5)
    B32 = O.uniform((256, 256), seed=6)
    C = cx.gemm(to_dev_f32(A32, dev), to_dev_f32(B32, dev))
    assert cx.last_kernel().startswith("gemm_f32_")
    assert np.array_equal(C.cpu().numpy(), O.gemm_f32(A32, B32))  # still the bit-exact FFMA chain


@pytest.mark.parametrize("variant,kernel", [("tc2", "gemm_tc2_256x256"), ("tc2_256x512", "gemm_tc2_256x512"),
                                            ("tc_128x256", "gemm_tc_128x256"),
                                            ("tc_128x128", "gemm_tc_128x128"), ("generic", "gemm_simt_generic")])
def test_forced_variant_runs_and_agrees(dev, table, variant, kernel):
    dt = O.F16
    M, N, K = 640, 520, 384
    A = O.to_lowp(O.normal((M, K), seed=3) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((K, N), seed=4), dt)
    ref = O.gemm_lowp(dt, A, B)
    tuning.force(variant)
    C = cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev))
    assert cx.last_kernel() == kernel
    assert O.max_relative(O.from_lowp(lowp_bits(C), dt), O.from_lowp(ref, dt)) <= 1e-2


def test_shipped_table_loads(table):
    if not tuning.DEFAULT_TABLE.exists():
        pytest.skip("no shipped table")
    assert tuning.load() >= 0  # loads (it may hold no rule where the built-in choice wins everywhere)
