"""at_gemv_t_static_scratch: the orientation-T GEMV for callers that cannot
allocate device memory (their memory belongs to another allocator, or they
cannot take cudaMalloc's device-wide synchronisation mid-loop). Its split-K
scratch is a static device array inside the library; the result must equal
at_gemv's within the GEMV tolerance, on two calls in a row (the array keeps
the previous call's contents). This file runs last so a failure here leaves
every other test already run."""
import numpy as np
import pytest
import torch

from auratensor_b200 import _lib, synth
from auratensor_b200.core import context, ptr
from auratensor_b200.quant import ORIENT_N, ORIENT_T, QMatrix
from oracle import ref

pytestmark = pytest.mark.gpu
TOL = 2e-5  # per output, times sum_i |w_i x_i| (the GEMV tests' bound)


def static_gemv(m, x, y):
    _lib.call("at_gemv_t_static_scratch", context(m.device), m._h, ptr(x), ptr(y), x.shape[0])


@pytest.mark.parametrize("qt", [ref.GGML_Q4_0, ref.GGML_Q8_0])
# The batch-8 cases that split a block column over CTAs and (16384, 64, 1)
# (each block column split over 16 CTAs) put their partials in the static
# array; the other splits combine in cluster shared memory, and (300, 640, 1)
# and (256, 8192, 8) do not split (the latter must not be rejected for
# partials it never writes).
@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 1), (2048, 1024, 2), (300, 640, 1), (1024, 512, 8),
                                             (8192, 64, 8), (16384, 64, 1), (256, 8192, 8)])
def test_static_scratch_matches_at_gemv(qt, rows, cols, batch, cuda):
    g = torch.Generator(device=cuda).manual_seed(rows + cols + batch)
    blocks = synth.generate_torch_tensor((rows, cols), qt, g, cuda)
    m = QMatrix(qt, ORIENT_T, rows, cols, blocks)
    W = ref.dequant(qt, blocks.cpu().numpy(), rows * cols).reshape(rows, cols).astype(np.float64)
    x = torch.randn((batch, rows), device=cuda)
    want = m.gemv(x).cpu().numpy()  # the existing entry point
    xd = x.cpu().numpy().astype(np.float64)
    exact = xd @ W  # the oracle's dequantized weights, in float64
    bound = TOL * (np.abs(xd) @ np.abs(W)) + 1e-30
    for _ in range(2):
        y = torch.full((batch, cols), float("nan"), device=cuda)
        static_gemv(m, x, y)
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.all(np.abs(got - want) <= bound)
        assert np.all(np.abs(got - exact) <= bound)


def test_static_scratch_rejects_oversized_split(cuda):
    # batch 8 over 16 block columns of 65536 rows splits each column over 22
    # CTAs (more than one cluster): 16 * 22 * 8 * 32 partials exceed the static 61440
    g = torch.Generator(device=cuda).manual_seed(1)
    m = QMatrix(ref.GGML_Q4_0, ORIENT_T, 65536, 512, synth.generate_torch_tensor((65536, 512), ref.GGML_Q4_0, g, cuda))
    x = torch.randn((8, 65536), device=cuda)
    y = torch.empty((8, 512), device=cuda)
    with pytest.raises(_lib.IllegalArgumentException, match="static maximum"):
        static_gemv(m, x, y)


def test_static_scratch_takes_orientation_t_only(cuda):
    g = torch.Generator(device=cuda).manual_seed(2)
    m = QMatrix(ref.GGML_Q4_0, ORIENT_N, 64, 64, synth.generate_torch_tensor((64, 64), ref.GGML_Q4_0, g, cuda))
    with pytest.raises(_lib.IllegalArgumentException, match="orientation-T"):
        static_gemv(m, torch.zeros((1, 64), device=cuda), torch.zeros((1, 64), device=cuda))
