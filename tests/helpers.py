"""Shared helpers for the GPU parity tests."""
from contextlib import contextmanager

import numpy as np
import torch

import oracle as O

TDT = {O.F16: torch.float16, O.BF16: torch.bfloat16}


def to_dev_f32(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)


def to_dev_lowp(bits: np.ndarray, dt: int, dev) -> torch.Tensor:
    """uint16 bit patterns -> device fp16/bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(TDT[dt])


def lowp_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().view(torch.int16).cpu().numpy().view(np.uint16)


def fp32_reference_gpu(A: torch.Tensor, B: torch.Tensor, transA=False, transB=False) -> torch.Tensor:
    """Plain fp32 (TF32 off) torch product of widened inputs on the GPU — used
    only for full-size checks where the CPU oracle would take minutes."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a = A.float().t() if transA else A.float()
        b = B.float().t() if transB else B.float()
        return a @ b
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@contextmanager
def forced_variant(name):
    """Run a block with one GEMM variant forced (cuopx_set_gemm_variant), so a
    parity test exercises that kernel whatever the size thresholds choose."""
    from cuop_b200 import tuning

    tuning.force(name)
    try:
        yield
    finally:
        tuning.force(None)

