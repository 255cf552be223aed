"""Level-1 vector ops (vector-ops plugin path) with standard BLAS semantics."""
import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [0, 1, 1000, 1 << 20, 3_000_017])
def test_reductions(dev, n):
    x32 = O.uniform(n, seed=1)
    y32 = O.uniform(n, seed=2)
    x = torch.from_numpy(x32).to(dev)
    y = torch.from_numpy(y32).to(dev)
    xd, yd = x32.astype(np.float64), y32.astype(np.float64)
    tol = 1e-5 * max(1.0, np.sqrt(n))
    assert abs(cx.dot(x, y).item() - xd @ yd) <= tol * max(1.0, np.abs(xd * yd).sum() / max(n, 1))
    assert abs(cx.asum(x).item() - np.abs(xd).sum()) <= 1e-6 * max(1.0, np.abs(xd).sum())
    assert abs(cx.nrm2(x).item() - np.sqrt((xd * xd).sum())) <= 1e-6 * max(1.0, np.sqrt((xd * xd).sum()))
    if n:
        assert cx.iamax(x).item() == int(np.argmax(np.abs(x32))) + 1
        assert cx.iamin(x).item() == int(np.argmin(np.abs(x32))) + 1
    else:
        assert cx.iamax(x).item() == 0


def test_iamax_first_index_on_ties(dev):
    x = torch.tensor([1.0, -5.0, 3.0, 5.0, -5.0], device=dev)
    assert cx.iamax(x).item() == 2
    assert cx.iamin(torch.tensor([2.0, -1.0, 1.0], device=dev)).item() == 2


def test_elementwise(dev):
    n = 100_003
    x32 = O.uniform(n, seed=3)
    y32 = O.uniform(n, seed=4)
    x = torch.from_numpy(x32).to(dev)
    y = torch.from_numpy(y32).to(dev)
    cx.axpy(2.5, x, y)
    np.testing.assert_allclose(y.cpu().numpy(), np.float32(2.5) * x32 + y32, rtol=1e-6, atol=1e-6)
    cx.scal(-0.5, y)
    z = torch.empty_like(x)
    cx.copy(y, z)
    assert torch.equal(z, y)
    a, b = x.clone(), y.clone()
    cx.swap(a, b)
    assert torch.equal(a, y) and torch.equal(b, x)
    c, s = 0.6, 0.8
    xr, yr = x.clone(), y.clone()
    cx.rot(xr, yr, c, s)
    xn, yn = x.cpu().numpy(), y.cpu().numpy()
    np.testing.assert_allclose(xr.cpu().numpy(), c * xn + s * yn, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(yr.cpu().numpy(), c * yn - s * xn, rtol=1e-6, atol=1e-6)


def test_strided_and_negative_increments(dev):
    x32 = O.uniform(30, seed=5)
    y32 = O.uniform(30, seed=6)
    x = torch.from_numpy(x32).to(dev)
    y = torch.from_numpy(y32).to(dev)
    d = cx.dot(x, y, n=10, incx=3, incy=-3).item()
    ref = np.dot(x32[0:30:3].astype(np.float64), y32[0:30:3][::-1].astype(np.float64))
    assert abs(d - ref) < 1e-5


def test_gather_column_blocks(dev):
    G, M, Nb = 4, 33, 24
    blocks = torch.arange(G * M * Nb, device=dev, dtype=torch.float32).view(G, M, Nb).to(torch.bfloat16)
    out = torch.empty(M, G * Nb, device=dev, dtype=torch.bfloat16)
    cx.gather_column_blocks(blocks, out)
    ref = torch.cat([blocks[g] for g in range(G)], dim=1)
    assert torch.equal(out, ref)


def test_copy_stages_through_pinned_host_memory(dev):
    """copy() with one side in pinned host memory reads or writes it directly."""
    x = torch.randn(10007).pin_memory()
    d = torch.empty(10007, device=dev)
    cx.copy(x, d)
    back = torch.full((10007,), float("nan")).pin_memory()
    cx.copy(d, back)
    torch.cuda.synchronize()
    assert torch.equal(back, x)
    with pytest.raises(cx.CuopError):
        cx.copy(torch.zeros(4), torch.zeros(4, device=dev))  # pageable host memory
    with pytest.raises(cx.CuopError):
        cx.copy(x, back)  # neither side on the device
