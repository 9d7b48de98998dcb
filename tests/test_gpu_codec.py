"""Block codecs and fp16 decode on the GPU vs the oracle and the reference KATs."""
import math

import numpy as np
import pytest
import torch

from auratensor_b200 import _lib, synth
from auratensor_b200.core import Fp16
from auratensor_b200.quant import Q4_0, Q8_0
from oracle import ref

pytestmark = pytest.mark.gpu


def test_fp16_all_bit_patterns(cuda, kats):
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).to(cuda)
    got = Fp16.toFloat(bits).cpu().numpy().view(np.uint32)
    want = ref.fp16_bits_to_f32(np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)).view(np.uint32)
    assert np.array_equal(got, want)
    for c in kats["fp16"]:
        assert int(got[c["bits"]]) == c["expect_bits"]


def test_q4_0_dequant_golden(cuda, kats):
    c = kats["q4_0_dequant"]
    src = torch.frombuffer(bytearray.fromhex(c["blocks_hex"]), dtype=torch.uint8).to(cuda)
    got = Q4_0.dequantToFloat(src, None, c["n"]).cpu().numpy()
    assert np.array_equal(got, np.array(c["expect"], dtype=np.float32))


def test_q4_0_dot_nan_scale(cuda, kats):
    c = kats["q4_0_dot_nan"]
    src = torch.frombuffer(bytearray.fromhex(c["blocks_hex"]), dtype=torch.uint8).to(cuda)
    x = torch.tensor(c["x"], dtype=torch.float32, device=cuda)
    assert math.isnan(Q4_0.dot(src, x, c["n"]))


@pytest.mark.parametrize("codec,qt", [(Q4_0, ref.GGML_Q4_0), (Q8_0, ref.GGML_Q8_0)])
@pytest.mark.parametrize("n", [32, 4096, 32 * 1000])
def test_dequant_and_dot_vs_oracle(cuda, codec, qt, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 0.02).astype(np.float32)
    blocks = synth.quantize(x, qt)
    src = torch.from_numpy(blocks).to(cuda)
    got = codec.dequantToFloat(src, None, n).cpu().numpy()
    want = ref.dequant(qt, blocks, n)
    assert np.array_equal(got, want)  # dequant is exact arithmetic: bit-identical
    v = rng.standard_normal(n).astype(np.float32)
    d = codec.dot(src, torch.from_numpy(v).to(cuda), n)
    w = float(np.dot(want.astype(np.float64), v.astype(np.float64)))
    assert abs(d - w) <= 1e-5 * float(np.sum(np.abs(want) * np.abs(v))) + 1e-12


def test_subnormal_scale_flushes(cuda):
    blk = bytes([0x01, 0x00]) + bytes([0xFF] * 16)  # d = smallest subnormal -> 0
    src = torch.frombuffer(bytearray(blk), dtype=torch.uint8).to(cuda)
    got = Q4_0.dequantToFloat(src, None, 32).cpu().numpy()
    assert np.all(got == 0)


def test_bad_lengths_raise(cuda):
    src = torch.zeros(18, dtype=torch.uint8, device=cuda)
    with pytest.raises(_lib.IllegalArgumentException):
        Q4_0.dequantToFloat(src, torch.empty(31, device=cuda), 31)
    out = Q4_0.dequantToFloat(src, torch.empty(1, device=cuda), 0)
    assert out.numel() == 1
