"""Tensor-core (tcgen05) prompt GEMM vs the oracle's dequantized FP32 product.

The GEMM rounds the dequantized weights and the activations to bf16 and sums
in FP32, so each output may differ from the FP32 oracle by about two bf16
roundings per product: the bound is 8e-3 x sum_k |w_k x_k| (2^-8 is the
relative error of a product of two bf16-rounded factors, plus margin); the
model-level prompt tolerance is 2e-2 of the logit range.
"""
import numpy as np
import pytest
import torch

from auratensor_b200 import synth
from auratensor_b200.quant import ORIENT_N, ORIENT_T, QMatrix
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 8e-3


def check(qt, orient, rows, cols, tokens, cuda, seed=0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    blocks = synth.quantize(w, qt)
    W = ref.dequant(qt, blocks, rows * cols).reshape(rows, cols).astype(np.float64)
    m = QMatrix(qt, orient, rows, cols, torch.from_numpy(blocks).to(cuda))
    n_in = cols if orient == ORIENT_N else rows
    x = rng.standard_normal((tokens, n_in)).astype(np.float32)
    y = m.gemm(torch.from_numpy(x).to(cuda)).cpu().numpy()
    Wo = W if orient == ORIENT_N else W.T  # [out][in]
    want = x.astype(np.float64) @ Wo.T
    bound = TOL * (np.abs(x).astype(np.float64) @ np.abs(Wo.T)) + 1e-30
    err = np.abs(y - want)
    assert np.all(err <= bound), (float(err.max()), float((err / bound).max()))


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("orient", [ORIENT_N, ORIENT_T])
@pytest.mark.parametrize("tokens", [1, 37, 128, 200, 256, 257, 300, 512, 513, 700, 1100])
def test_gemm_tc_small(qt, orient, tokens, cuda):
    """Above 256 tokens a CTA takes two 256-token tiles per weight tile (two
    TMEM accumulators); a last CTA row may hold one tile (513, 700) or two
    (1100: 512 + 512 + 76)."""
    check(qt, orient, 256, 128, tokens, cuda, seed=tokens)


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
@pytest.mark.parametrize("orient,rows,cols", [(ORIENT_N, 300, 640), (ORIENT_N, 1000, 256), (ORIENT_T, 640, 416),
                                              (ORIENT_T, 4096, 1024), (ORIENT_N, 16384, 128)])
@pytest.mark.parametrize("tokens", [130, 450])
def test_gemm_tc_ragged(qt, orient, rows, cols, tokens, cuda):
    """Ragged edges; the K steps of all tiles are split evenly over the SMs,
    so some tiles are summed from pieces of several CTAs (300 x 640: ten one-
    step pieces per tile) and some are whole inside one CTA (16384 x 128);
    450 tokens run the two-tile CTAs."""
    check(qt, orient, rows, cols, tokens, cuda, seed=rows + cols)


@pytest.mark.parametrize("orient,rows,cols", [(ORIENT_N, 2048, 1024), (ORIENT_T, 1024, 2048)])
def test_gemm_tc_repeatable(orient, rows, cols, cuda):
    """Pieces of a split tile are summed in K order by whichever CTA finishes
    last: the result does not depend on the arrival order."""
    rng = np.random.default_rng(5)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    m = QMatrix(ref.GGML_Q4_0, orient, rows, cols, torch.from_numpy(synth.quantize(w, ref.GGML_Q4_0)).to(cuda))
    n_in = cols if orient == ORIENT_N else rows
    x = torch.from_numpy(rng.standard_normal((400, n_in)).astype(np.float32)).to(cuda)
    first = m.gemm(x).cpu()
    for _ in range(5):
        assert torch.equal(m.gemm(x).cpu(), first)
