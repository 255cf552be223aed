"""The allocation-free GEMV entry point (cuopx_gemv_noalloc).

It is meant for callers that may not allocate device memory while running
(plugin hosts that own all device memory; serving loops where an allocation
could stall or fail), so it takes its split-K scratch from a fixed 2 MiB array
inside libcuopx.so instead of a caller workspace.  These tests call it
through the C ABI and compare it with cuopx_gemv, which runs the same
kernels with a caller-provided workspace, on two calls in a row with
different inputs: the second call must not see anything left in the shared
scratch by the first.  Both entry points run the same deterministic kernels,
so their results must be identical bit for bit; each is also checked against
the oracle (the CPU restatement of the reference's GEMV) within
||y - y_ref||_F / ||y_ref||_F <= 1e-5*sqrt(N).

This file is collected last on purpose (test_zz_*), so a run that stops at
the first failure has run every other test before it.
"""
import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from cuop_b200 import _native as N
from helpers import to_dev_f32

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _noalloc(A, x, y, trans, M, Nn, lda, alpha=1.0, beta=0.0, dtype=N.F32):
    return N.lib().cuopx_gemv_noalloc(dtype, int(trans), M, Nn, alpha, A.data_ptr(), lda, x.data_ptr(), beta,
                                      y.data_ptr(), _stream())


def _with_workspace(A, x, y, trans, M, Nn, lda, alpha=1.0, beta=0.0, dtype=N.F32):
    need = N.lib().cuopx_gemv_workspace_size(dtype, int(trans), M, Nn)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=A.device)
    rc = N.lib().cuopx_gemv(dtype, int(trans), M, Nn, alpha, A.data_ptr(), lda, x.data_ptr(), beta, y.data_ptr(),
                            ws.data_ptr(), ws.numel(), _stream())
    torch.cuda.synchronize()
    return rc


# (M, N, trans, kernel the split-K scratch is used by)
CASES = [
    (8192, 8192, True, "gemv_t_lsu"),       # streaming transposed kernel, split partials in scratch
    (16, 262144, False, "gemv_n_splitk"),   # short-wide plain GEMV, split partials in scratch
]


@pytest.mark.parametrize("M,Nn,trans,kernel", CASES)
def test_noalloc_matches_workspace_entry_point_twice(dev, M, Nn, trans, kernel):
    tol = 1e-5 * np.sqrt(Nn)
    for call, seed in enumerate((101, 202)):  # two calls in a row, different data
        A32 = O.uniform((Nn, M) if trans else (M, Nn), seed=seed)
        x32 = O.uniform(Nn, seed=seed + 1)
        y032 = O.uniform(M, seed=seed + 2)
        A, x = to_dev_f32(A32, dev), to_dev_f32(x32, dev)
        lda = M if trans else Nn
        y_ref = to_dev_f32(y032, dev)
        assert _with_workspace(A, x, y_ref, trans, M, Nn, lda, alpha=1.5, beta=-0.25) == N.SUCCESS
        y = to_dev_f32(y032, dev)
        assert _noalloc(A, x, y, trans, M, Nn, lda, alpha=1.5, beta=-0.25) == N.SUCCESS
        assert cx.last_kernel() == kernel, (call, cx.last_kernel())
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), call
        cpu = O.gemv_f32(A32, x32, y032, trans=trans, alpha=1.5, beta=-0.25)
        err = O.rel_frobenius(y.cpu().numpy(), cpu)
        assert err <= tol, (call, err)


def test_noalloc_rejects_scratch_beyond_limit(dev):
    """bf16 transposed GEMV whose rows are not a multiple of 16 bytes (M = 8191)
    runs the generic split kernel, which needs more than the 2 MiB scratch."""
    M, Nn = 8191, 8192
    need = N.lib().cuopx_gemv_workspace_size(N.BF16, 1, M, Nn)
    assert need > (2 << 20)
    A = torch.zeros(Nn, M, dtype=torch.bfloat16, device=dev)
    x = torch.zeros(Nn, dtype=torch.bfloat16, device=dev)
    y = torch.full((M,), 7.0, dtype=torch.bfloat16, device=dev)
    rc = _noalloc(A, x, y, True, M, Nn, M, dtype=N.BF16)
    assert rc == N.RESOURCE_UNAVAILABLE
    torch.cuda.synchronize()
    assert torch.all(y == 7.0)  # nothing was launched


def test_noalloc_streaming_transposed_fits_at_any_size(dev):
    """The streaming transposed kernel's partials are bounded by the resident
    CTA count times one strip, so even bf16 8192^2 fits the scratch."""
    M = Nn = 8192
    A = torch.randn(Nn, M, device=dev).bfloat16()
    x = torch.randn(Nn, device=dev).bfloat16()
    y_ref = torch.empty(M, dtype=torch.bfloat16, device=dev)
    assert _with_workspace(A, x, y_ref, True, M, Nn, M, dtype=N.BF16) == N.SUCCESS
    y = torch.empty(M, dtype=torch.bfloat16, device=dev)
    assert _noalloc(A, x, y, True, M, Nn, M, dtype=N.BF16) == N.SUCCESS
    assert cx.last_kernel() == "gemv_t_lsu"
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
