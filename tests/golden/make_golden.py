"""Writes tests/golden/reference_kats.json: the known-answer cases the
reference's JUnit suite holds for the decode path, restated as data.

No JDK exists where these fixtures were produced, so each case rebuilds the
inputs exactly as the reference test constructs them (java.util.Random
sequences, float casts) and records the expected values the test asserts
(file:line of each test under src/test/java/io/auratensor/). Run:

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import os
import struct
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.java_random import JavaRandom  # noqa: E402


def f32(v: float) -> float:
    return float(np.float32(v))


def f32_bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


def fp16_cases():
    # core/Fp16Test.java:10-48: bit pattern -> expected float (bits of the result)
    return [
        {"bits": 0x0000, "expect_bits": 0x00000000},   # :11 zeroIsZero
        {"bits": 0x3C00, "expect_bits": 0x3F800000},   # :17 one
        {"bits": 0x4000, "expect_bits": 0x40000000},   # :24 two
        {"bits": 0x8000, "expect_bits": 0x80000000},   # :29-32 negative zero keeps its sign
        {"bits": 0x7C00, "expect_bits": 0x7F800000},   # :38 +inf
        {"bits": 0xFC00, "expect_bits": 0xFF800000},   # :40 -inf
        {"bits": 0x0001, "expect_bits": 0x00000000},   # :46 subnormal flushes to zero
        {"bits": 0x0200, "expect_bits": 0x00000000},   # :47
    ]


def q4_dequant_case():
    # quant/Q4_0Test.java:15-51 dequantReferenceMatches: 128 elements, Random(7)
    r = JavaRandom(7)
    blocks = bytearray()
    for _ in range(4):
        scale = f32(r.next_gaussian() * 0.05)
        half = ((f32_bits(scale) >> 13) & 0x7FF) | 0x3C00
        blk = bytearray(struct.pack("<H", half & 0xFFFF))
        for _ in range(16):
            lo = r.next_int(16)
            hi = r.next_int(16)
            blk.append(((hi << 4) | lo) & 0xFF)
        blocks += blk
    # expected: (q - 8) * Fp16.toFloat(half), q from the interleaved nibble order (:41-47)
    from oracle.ref import fp16_bits_to_f32
    expect = []
    for b in range(4):
        half = blocks[b * 18] | (blocks[b * 18 + 1] << 8)
        scale = float(fp16_bits_to_f32(np.array([half], dtype=np.uint16))[0])
        for i in range(32):
            packed = blocks[b * 18 + 2 + i // 2]
            q = (packed & 0xF) if i % 2 == 0 else ((packed >> 4) & 0xF)
            expect.append(f32((q - 8) * scale))
    return {"n": 128, "blocks_hex": blocks.hex(), "expect": expect, "tol": 1e-3}


def q4_dot_case():
    # quant/Q4_0Test.java:53-92 fusedDotMatchesScalar: Random(101), scale 0.05f
    # encoded as (bits >>> 13) | 0x3C00, which truncates to 0xFE66 = NaN (the
    # test compares NaN with NaN). Expected dot: NaN.
    r = JavaRandom(101)
    half = ((f32_bits(f32(0.05)) >> 13) | 0x3C00) & 0xFFFF
    blocks = bytearray()
    for _ in range(8):
        blk = bytearray(struct.pack("<H", half))
        for _ in range(16):
            lo = r.next_int(16)
            hi = r.next_int(16)
            blk.append(((hi << 4) | lo) & 0xFF)
        blocks += blk
    w = [f32(f32(r.next_float()) - f32(0.5)) for _ in range(256)]
    return {"n": 256, "half": half, "blocks_hex": blocks.hex(), "x": w, "expect_nan": True}


def kernels_cases():
    # core/KernelsTest.java
    x16 = [f32(math.sin(i) * 2 + 0.5) for i in range(16)]                  # :33
    w16 = [f32(f32(math.cos(i * 0.01)) + f32(1.0)) for i in range(16)]       # :34
    silu_x = [f32(f32(float(i - 16)) * f32(0.3)) for i in range(32)]        # :51
    silu_expect = [f32(v / f32(1.0 + f32(math.exp(-v)))) for v in silu_x]  # :54-55
    sm_x = [f32(i * 0.7 - 2) for i in range(8)]                             # :67
    mx = max(sm_x)
    e = [f32(math.exp(f32(v - mx))) for v in sm_x]                           # :72-75
    s = f32(0.0)
    for v in e:
        s = f32(s + v)
    sm_expect = [f32(v / s) for v in e]                                      # :77
    sum_x = [f32(i * 0.13 - 4) for i in range(64)]                          # :88
    rope_x = [f32(f32(float(i + 1)) * f32(0.3)) for i in range(8)]          # :98
    cos_r, sin_r = [], []
    for i in range(4):                                                      # :106-114
        a = f32(f32(float(i)) * f32(0.7))
        cos_r += [f32(math.cos(a))] * 2
        sin_r += [f32(math.sin(a))] * 2
    M, K, N = 4, 16, 6                                                      # :134-143
    A = [[float((i + 1) * (k + 1)) for k in range(K)] for i in range(M)]
    B = [[float((k + 2) * (j + 3)) for j in range(N)] for k in range(K)]
    C = [[sum(A[i][k] * B[k][j] for k in range(K)) for j in range(N)] for i in range(M)]
    Mv, Kv = 8, 32                                                          # :167-174
    Av = [[float((i + 1) * (k + 1)) for k in range(Kv)] for i in range(Mv)]
    xv = [f32(f32(0.1) * f32(float(k + 1))) for k in range(Kv)]
    yv = []
    for i in range(Mv):
        acc = f32(0.0)
        for k in range(Kv):
            acc = f32(acc + f32(Av[i][k] * xv[k]))
        yv.append(acc)
    return {
        "rmsnorm": {"x": x16, "w": w16, "eps": 1e-5, "tol": 1e-5},
        "silu": {"x": silu_x, "expect": silu_expect, "tol": 1e-5},
        "softmax": {"x": sm_x, "expect": sm_expect, "tol": 1e-5},
        "softmax_sum": {"x": sum_x, "expect_sum": 1.0, "tol": 1e-4},
        "rope_invertible": {"x": rope_x, "cos": cos_r, "sin": sin_r, "head_dim": 8, "tol": 1e-5},
        "sgemm": {"M": M, "K": K, "N": N, "A": A, "B": B, "expect": C, "tol": 1e-3},
        "sgemv": {"M": Mv, "K": Kv, "A": Av, "x": xv, "expect": yv, "tol": 1e-3},
    }


def sampler_cases():
    # inference/SamplerTest.java; config = [temperature, topK, topP, repetitionPenalty, seed]
    top_k_one = [1000.0 if i == 42 else float(i) for i in range(100)]
    top_p = [-100.0] * 1024
    top_p[100] = 0.0
    top_p[101] = -5.0
    return [
        {"name": "greedyPicksArgmax", "logits": [0.1, 0.5, 0.7, 0.3, 0.2], "history": None,
         "config": [1.0, 1, 1.0, 1.0, 0], "expect": [2]},                                   # :10-14
        {"name": "tempZeroIsGreedy", "logits": [0.1, 0.5, 0.7, 0.3], "history": None,
         "config": [0.0, 1, 1.0, 1.0, 0], "expect": [2]},                                   # :17-21
        {"name": "topKOneIsGreedy", "logits": top_k_one, "history": None,
         "config": [1.0, 1, 1.0, 1.0, 0], "expect": [42]},                                  # :24-29
        {"name": "repetitionPenaltyReducesSeenTokens", "logits": [1.0, 1.0, 1.0, 1.0], "history": [0, 1],
         "config": [1.0, 1, 1.0, 2.0, 42], "expect": [2, 3]},                                # :32-40
        {"name": "topPStillPicksFromAllowedSet", "logits": top_p, "history": None,
         "config": [1.0, 1024, 0.999, 1.0, 7], "expect": [100, 101], "first": 100},          # :43-56
        {"name": "eosTokenIsRespected", "logits": [-1e9, 0.0, -1e9, -1e9], "history": [2],
         "config": [1.0, 1, 1.0, 1.0, 0], "expect": [1]},                                   # :59-65
    ]


def gguf_minimal_header_hex():
    # format/GgufFileTest.java:22-75: v3, 0 tensors, 1 KV general.architecture="llama",
    # tightly packed, file length rounded up to 32
    b = struct.pack("<IIQQ", 0x46554747, 3, 0, 1)
    b += struct.pack("<q", 20) + b"general.architecture" + struct.pack("<i", 8) + struct.pack("<q", 5) + b"llama"
    b += b"\0" * ((-len(b)) % 32)
    return b.hex()


def q6_k_cases():
    # quant/Q6_KTest.java: dequantMatchesCanonicalInnerLoop (:22-104, Random(7),
    # d = Float.floatToFloat16(0.04f)), zeroBiasProducesAllZero (:106-131) and
    # q0MinAndQ63MaxProducedSignExtreme (:133-181). Expected values follow the
    # test's restatement of the canonical loop: (d * scale) * (q - 32) in float.
    def block(ql, qh, sc, d16):
        return bytes(ql) + bytes(qh) + bytes((v & 0xFF) for v in sc) + struct.pack("<H", d16)

    def expect(blk):
        d16 = blk[208] | (blk[209] << 8)
        d = float(np.array([d16], dtype=np.uint16).view(np.float16)[0])
        out = [0.0] * 256
        for n in (0, 128):
            for l in range(32):
                is_ = l // 16
                lo, hi, qh = blk[n // 2 + l], blk[n // 2 + l + 32], blk[128 + n // 4 + l]
                s = [np.int8(np.uint8(blk[192 + n // 16 + is_ + 2 * j])) for j in range(4)]
                q = [((lo & 0xF) | (((qh >> 0) & 3) << 4)) - 32, ((hi & 0xF) | (((qh >> 2) & 3) << 4)) - 32,
                     (((lo >> 4) & 0xF) | (((qh >> 4) & 3) << 4)) - 32, (((hi >> 4) & 0xF) | (((qh >> 6) & 3) << 4)) - 32]
                for j in range(4):
                    out[n + l + 32 * j] = f32(np.float32(np.float32(d) * np.float32(s[j])) * np.float32(q[j]))
        return out

    r = JavaRandom(7)
    d16 = int(np.array([np.float16(np.float32(0.04))]).view(np.uint16)[0])
    sc = [r.next_int(241) - 120 for _ in range(16)]
    ql = []
    for _ in range(128):
        lo = r.next_int(16)
        hi = r.next_int(16)
        ql.append(((hi << 4) | lo) & 0xFF)
    qh = []
    for _ in range(64):
        b0, b1, b2, b3 = r.next_int(4), r.next_int(4), r.next_int(4), r.next_int(4)
        qh.append(b0 | (b1 << 2) | (b2 << 4) | (b3 << 6))
    canon = block(ql, qh, sc, d16)
    zero = block([0] * 128, [0xAA] * 64, [1] * 16, 0x3C00)
    qmax = block([0xFF] * 128, [0xFF] * 64, [1] * 16, 0x3C00)
    qmin = block([0] * 128, [0] * 64, [1] * 16, 0x3C00)
    return [{"name": "canonical_random7", "block_hex": canon.hex(), "expect": expect(canon)},
            {"name": "zero_bias", "block_hex": zero.hex(), "expect": [0.0] * 256},
            {"name": "q63_max", "block_hex": qmax.hex(), "expect": [31.0] * 256},
            {"name": "q0_min", "block_hex": qmin.hex(), "expect": [-32.0] * 256}]


def main():
    out = {
        "source": "restated from the reference JUnit tests (src/test/java/io/auratensor)",
        "fp16": fp16_cases(),
        "q4_0_dequant": q4_dequant_case(),
        "q4_0_dot_nan": q4_dot_case(),
        "q6_k_dequant": q6_k_cases(),
        "kernels": kernels_cases(),
        "sampler": sampler_cases(),
        "gguf_minimal_header_hex": gguf_minimal_header_hex(),
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(path)


if __name__ == "__main__":
    main()
