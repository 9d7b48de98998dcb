"""core/KernelsTest.java on the GPU: the reference's formula cases plus the oracle."""
import numpy as np
import pytest
import torch

from auratensor_b200 import _lib
from auratensor_b200.core import DType, Kernels, Tensor
from oracle import ref

pytestmark = pytest.mark.gpu


def T(values, cuda, shape=None):
    a = np.asarray(values, dtype=np.float32)
    t = Tensor.allocate(DType.FP32, *(shape or a.shape))
    t.data().copy_(torch.from_numpy(a.reshape(-1)).to(cuda))
    return t


def host(t):
    return t.data().cpu().numpy()


def test_rmsnorm(cuda, kats):
    k = kats["kernels"]["rmsnorm"]
    x, w = T(k["x"], cuda), T(k["w"], cuda)
    Kernels.rmsNormInPlace(x, w, k["eps"])
    want = np.array(k["x"], dtype=np.float32)
    ref.rmsnorm_inplace(want, np.array(k["w"], dtype=np.float32), k["eps"])
    np.testing.assert_allclose(host(x), want, rtol=0, atol=k["tol"])


def test_rmsnorm_rank2_and_checks(cuda):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 4096)).astype(np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    x = T(a, cuda)
    Kernels.rmsNormInPlace(x, T(w, cuda), 1e-5)
    want = a.copy()
    ref.rmsnorm_inplace(want, w, 1e-5)
    np.testing.assert_allclose(host(x).reshape(3, -1), want, rtol=2e-6, atol=1e-6)
    with pytest.raises(_lib.IllegalArgumentException):
        Kernels.rmsNormInPlace(x, T(w[:10], cuda), 1e-5)


def test_silu(cuda, kats):
    k = kats["kernels"]["silu"]
    x = T(k["x"], cuda)
    Kernels.siluInPlace(x)
    np.testing.assert_allclose(host(x), k["expect"], rtol=0, atol=k["tol"])


def test_softmax(cuda, kats):
    k = kats["kernels"]["softmax"]
    x = T(k["x"], cuda)
    Kernels.softmaxInPlace(x)
    np.testing.assert_allclose(host(x), k["expect"], rtol=0, atol=k["tol"])
    s = kats["kernels"]["softmax_sum"]
    y = T(s["x"], cuda)
    Kernels.softmaxInPlace(y)
    assert abs(float(host(y).sum()) - 1.0) < s["tol"]


def test_rope_invertible_and_oracle(cuda, kats):
    r = kats["kernels"]["rope_invertible"]
    x, c, s = T(r["x"], cuda), T(r["cos"], cuda), T(r["sin"], cuda)
    Kernels.ropeInPlace(x, c, s, r["head_dim"])
    want = np.array(r["x"], dtype=np.float32)
    ref.rope_inplace(want, np.array(r["cos"], np.float32), np.array(r["sin"], np.float32), 8)
    np.testing.assert_allclose(host(x), want, rtol=0, atol=1e-6)
    Kernels.ropeInPlace(x, c, T(-np.array(r["sin"]), cuda), r["head_dim"])
    np.testing.assert_allclose(host(x), r["x"], atol=r["tol"])
    with pytest.raises(_lib.IllegalArgumentException):
        Kernels.ropeInPlaceSegment(x.data(), c.data(), s.data(), 3, 8)


def test_sgemm_and_sgemv(cuda, kats):
    g = kats["kernels"]["sgemm"]
    A, B = T(g["A"], cuda), T(g["B"], cuda)
    C = Tensor.allocate2D(DType.FP32, g["M"], g["N"])
    Kernels.sgemm(A, B, C)
    np.testing.assert_allclose(host(C).reshape(g["M"], g["N"]), g["expect"], atol=g["tol"])
    v = kats["kernels"]["sgemv"]
    A, x = T(v["A"], cuda), T(v["x"], cuda)
    y = Tensor.allocate1D(DType.FP32, v["M"])
    Kernels.sgemv(A, x, y)
    np.testing.assert_allclose(host(y), v["expect"], rtol=1e-6, atol=v["tol"])
    with pytest.raises(_lib.IllegalArgumentException):
        Kernels.sgemv(A, y, x)
