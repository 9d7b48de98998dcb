"""Fused-dequant GEMV (orientation N and T, Q4_0 and Q8_0, batch 1..8) vs the oracle.

Tolerance: the oracle's FP32 matvec over the dequantized weights and the
kernel differ only in summation order, so each output must agree within
2e-5 x sum_i |w_i x_i| (far below the 1e-3-of-logit-range model tolerance).
"""
import numpy as np
import pytest
import torch

from auratensor_b200 import _lib, synth
from auratensor_b200.quant import ORIENT_N, ORIENT_T, QMatrix
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 2e-5


def make(qt, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    blocks = synth.quantize(w, qt)
    return blocks, ref.dequant(qt, blocks, rows * cols).reshape(rows, cols)


def check(qt, orient, rows, cols, batch, cuda, seed=0):
    blocks, W = make(qt, rows, cols, seed)
    m = QMatrix(qt, orient, rows, cols, torch.from_numpy(blocks).to(cuda))
    rng = np.random.default_rng(seed + 1)
    n_in = cols if orient == ORIENT_N else rows
    x = rng.standard_normal((batch, n_in)).astype(np.float32)
    y = m.gemv(torch.from_numpy(x).to(cuda)).cpu().numpy()
    Wo = W if orient == ORIENT_N else W.T
    want = (x.astype(np.float64) @ Wo.T.astype(np.float64))
    bound = TOL * (np.abs(x).astype(np.float64) @ np.abs(Wo.T).astype(np.float64)) + 1e-30
    err = np.abs(y - want)
    assert np.all(err <= bound), (float(err.max()), float((err / bound).max()))
    return m, blocks


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("orient", [ORIENT_N, ORIENT_T])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8])
def test_small_shapes(qt, orient, batch, cuda):
    for rows, cols in [(64, 96), (1000, 256), (33, 32), (4096, 2048)]:
        check(qt, orient, rows, cols, batch, cuda, seed=rows + cols + batch)


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("shape", [(2048, 2048), (8192, 2048), (2048, 8192), (14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("batch", [1, 8])
def test_kernel_sweep_shapes(qt, shape, batch, cuda):
    """The kernel-sweep shapes (rows = out x cols = in), orientation N."""
    check(qt, ORIENT_N, shape[0], shape[1], batch, cuda, seed=7)


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("orient,rows,cols", [(ORIENT_N, 16, 14336), (ORIENT_N, 40, 8192), (ORIENT_N, 128, 4096),
                                              (ORIENT_T, 14336, 64), (ORIENT_T, 16, 14336), (ORIENT_T, 4096, 6144)])
@pytest.mark.parametrize("batch", [1, 2])
def test_segments_shared_by_many_ctas(qt, orient, rows, cols, batch, cuda):
    """Row groups (N) or block columns (T) whose tiles are spread over many
    CTAs: their partials meet in global scratch and the last CTA to arrive
    finishes them. Two calls in a row also check that the arrival counters
    are reset."""
    for seed in (11, 12):
        check(qt, orient, rows, cols, batch, cuda, seed=seed)


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("orient", [ORIENT_N, ORIENT_T])
def test_planar_relayout_is_lossless(qt, orient, cuda):
    blocks, _ = make(qt, 300, 640, 3)
    m = QMatrix(qt, orient, 300, 640, torch.from_numpy(blocks).to(cuda))
    assert np.array_equal(m.export_blocks().cpu().numpy(), blocks)
    m2 = QMatrix(qt, orient, 300, 640, blocks)  # host upload path
    assert np.array_equal(m2.export_blocks().cpu().numpy(), blocks)


def test_lm_head_columns_at_full_size(cuda):
    """128256 x 4096 Q4_0: W e_k is column k of the dequantized matrix (checked per column)."""
    rows, cols = 128256, 4096
    g = torch.Generator(device=cuda).manual_seed(5)
    blocks = synth.generate_torch_tensor((rows, cols), ref.GGML_Q4_0, g, cuda)
    m = QMatrix(ref.GGML_Q4_0, ORIENT_N, rows, cols, blocks)
    raw = blocks.cpu().numpy().reshape(rows, cols // 32, 18)
    for k in (0, 31, 2049, 4095):
        x = torch.zeros((1, cols), device=cuda)
        x[0, k] = 1.0
        y = m.gemv(x).cpu().numpy()[0]
        col = ref.q4_0_dequant(np.ascontiguousarray(raw[:, k // 32, :]), rows * 32).reshape(rows, 32)[:, k % 32]
        assert np.array_equal(y, col)
    # linearity on the full matrix: W(a + b) = Wa + Wb within FP32 rounding
    a = torch.randn((2, cols), device=cuda)
    ya, yb = m.gemv(a[:1]), m.gemv(a[1:])
    yab = m.gemv(a[:1] + a[1:])
    assert torch.allclose(yab, ya + yb, rtol=1e-4, atol=1e-4)


def test_nan_scale_propagates(cuda):
    blocks, _ = make(ref.GGML_Q4_0, 8, 64, 1)
    b = blocks.copy().reshape(8, 2, 18)
    b[3, 1, 0:2] = [0x66, 0xFE]  # NaN scale in row 3
    m = QMatrix(ref.GGML_Q4_0, ORIENT_N, 8, 64, b.reshape(-1))
    y = m.gemv(torch.ones((1, 64), device=cuda)).cpu().numpy()[0]
    assert np.isnan(y[3]) and np.all(np.isfinite(np.delete(y, 3)))


def test_gemv_arg_checks(cuda):
    blocks, _ = make(ref.GGML_Q4_0, 8, 64, 1)
    with pytest.raises(_lib.IllegalArgumentException):
        QMatrix(ref.GGML_Q4_0, ORIENT_N, 8, 60, blocks)
    m = QMatrix(ref.GGML_Q4_0, ORIENT_N, 8, 64, blocks)
    with pytest.raises(_lib.IllegalArgumentException):
        m.gemv(torch.ones((9, 64), device=cuda))
