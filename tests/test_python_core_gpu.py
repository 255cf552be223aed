"""The reference's Python operator classes (python/cuop/core.cpp names) on
the sm_100a kernels, through `cuop_b200.cuop`: the reference's known answers
(test_gemm.cpp, test_gemv.cpp, test_matmul.cpp) and seeded checks against
numpy / the oracle."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())


@pytest.fixture(scope="module")
def cuop():
    from cuop_b200 import build

    build.build()
    from cuop_b200 import cuop as m

    assert m.is_cuda_available()
    return m


def test_gemm_float_known_answer(cuop):
    g = GOLD["gemm_2x3x4"]
    A = cuop.tensor(np.array(g["A"], np.float32).reshape(g["M"], g["K"]))
    W = cuop.tensor(np.array(g["B"], np.float32).reshape(g["K"], g["N"]))
    C = cuop.zeros([g["M"], g["N"]])
    gemm = cuop.GemmFloat()
    gemm.set_weight(W)
    gemm.forward(A, C)
    np.testing.assert_allclose(C.to_numpy().ravel(), g["expected"], atol=g["tol"])
    assert repr(C) == "TensorFloat(2, 4)" and C.shape() == [2, 4] and C.size() == 8


def test_gemv_float_known_answer(cuop):
    g = GOLD["gemv_2x3"]
    A = cuop.tensor(np.array(g["A"], np.float32).reshape(g["M"], g["N"]))
    x = cuop.tensor(np.array(g["x"], np.float32))
    y = cuop.zeros([g["M"]])
    gemv = cuop.GemvFloat()
    gemv.set_weight(x)
    gemv.forward(A, y)
    np.testing.assert_allclose(y.to_numpy(), g["expected"], atol=g["tol"])


def test_matmul_and_batchmatmul_known_answers(cuop):
    g2, g3 = GOLD["matmul_2d"], GOLD["matmul_batch3d"]
    C = cuop.TensorFloat()
    cuop.MatMulFloat().forward(cuop.tensor(np.array(g2["A"], np.float32).reshape(g2["M"], g2["K"])),
                               cuop.tensor(np.array(g2["B"], np.float32).reshape(g2["K"], g2["N"])), C, -1)
    np.testing.assert_allclose(C.to_numpy().ravel(), g2["expected"], atol=g2["tol"])
    A3 = cuop.tensor(np.array(g3["A"], np.float32).reshape(g3["batch"], g3["M"], g3["K"]))
    B3 = cuop.tensor(np.array(g3["B"], np.float32).reshape(g3["batch"], g3["K"], g3["N"]))
    C3 = cuop.TensorFloat()
    cuop.BatchMatMulFloat().forward(A3, B3, C3)
    np.testing.assert_allclose(C3.to_numpy().ravel(), np.array(g3["expected"]).ravel(), atol=g3["tol"])


def test_vector_operators(cuop):
    x0 = O.uniform(10007, seed=1)
    y0 = O.uniform(10007, seed=2)
    x, y = cuop.tensor(x0), cuop.tensor(y0)
    assert abs(cuop.DotFloat().forward(x, y) - float(np.dot(x0.astype(np.float64), y0))) < 1e-3
    cuop.AxpyFloat(2.0).forward(x, y)
    cuop.ScalFloat(0.5).forward(y)
    z = cuop.zeros([10007])
    cuop.CopyFloat().forward(y, z)
    np.testing.assert_array_equal(z.to_numpy(), 0.5 * (2.0 * x0 + y0))


def test_jit_gemm_matches_operator(cuop):
    A0, W0 = O.uniform((257, 300), seed=3), O.uniform((300, 129), seed=4)
    A, W = cuop.tensor(A0), cuop.tensor(W0)
    C1, C2 = cuop.zeros([257, 129]), cuop.zeros([257, 129])
    gemm = cuop.GemmFloat(False, False, 1.0, 0.0)
    gemm.set_weight(W)
    gemm.forward(A, C1)
    jit = cuop.JITGemmFloat(gemm)
    jit.set_jit_config(cuop.get_default_jit_config())
    jit.enable_jit(True)
    assert jit.is_jit_compiled()
    jit.forward(A, C2)
    np.testing.assert_array_equal(C1.to_numpy(), C2.to_numpy())
    assert jit.get_performance_profile().kernel_name  # the plugin ran
    ref = A0.astype(np.float64) @ W0
    assert O.rel_frobenius(C1.to_numpy(), ref) <= 1e-5 * np.sqrt(300)


def test_double_and_errors(cuop):
    A0, W0 = np.random.default_rng(0).standard_normal((64, 48)), np.random.default_rng(1).standard_normal((48, 32))
    A, W = cuop.TensorDouble(), cuop.TensorDouble()
    A.copy_from(A0)
    W.copy_from(W0)
    C = cuop.TensorDouble([64, 32], 0.0)
    g = cuop.GemmDouble()
    g.set_weight(W)
    g.forward(A, C)
    np.testing.assert_allclose(C.to_numpy(), A0 @ W0, rtol=1e-12, atol=1e-12)
    bad = cuop.zeros([3, 3])
    with pytest.raises(RuntimeError):
        g2 = cuop.GemmFloat()
        g2.set_weight(cuop.zeros([4, 4]))
        g2.forward(bad, cuop.zeros([3, 4]))  # K mismatch: SHAPE_MISMATCH -> RuntimeError
    with pytest.raises(RuntimeError):
        cuop.DotDouble().forward(cuop.TensorDouble([4]), cuop.TensorDouble([4]))  # fp64 vector ops: unsupported


def test_randn_is_normal_and_seeded(cuop):
    t = cuop.randn([256, 512], 0.5, 2.0, seed=7)
    a = t.to_numpy()
    assert a.shape == (256, 512)
    assert abs(a.mean() - 0.5) < 0.05 and abs(a.std() - 2.0) < 0.05
    np.testing.assert_array_equal(cuop.randn([256, 512], 0.5, 2.0, seed=7).to_numpy(), a)
    assert not np.array_equal(cuop.randn([256, 512], 0.5, 2.0, seed=8).to_numpy(), a)
    assert cuop.randn([3]).size() == 3
