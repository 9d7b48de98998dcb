"""The oracle pinned against the reference's own known-answer tests (CPU)."""
import math

import numpy as np
import pytest

from oracle import ref
from oracle.java_random import JavaRandom


def test_java_random_published_value():
    # java.util.Random(42).nextInt() is the documented LCG's first output
    assert JavaRandom(42).next_int() == -1170105035


def test_fp16_kats(kats):
    for c in kats["fp16"]:
        got = ref.fp16_bits_to_f32(np.array([c["bits"]], dtype=np.uint16)).view(np.uint32)[0]
        assert int(got) == c["expect_bits"], hex(c["bits"])


def test_fp16_nan_and_normals():
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    out = ref.fp16_bits_to_f32(bits)
    e = (bits >> 10) & 0x1F
    m = bits & 0x3FF
    normal = (e > 0) & (e < 31)
    # normals agree with IEEE half conversion; subnormals flush to signed zero
    assert np.array_equal(out[normal], bits[normal].view(np.float16).astype(np.float32))
    sub = e == 0
    assert np.all(out[sub] == 0) and np.array_equal(np.signbit(out[sub]), (bits[sub] >> 15) == 1)
    assert np.all(np.isnan(out[(e == 31) & (m != 0)]))


def test_q4_0_dequant_golden(kats):
    c = kats["q4_0_dequant"]
    got = ref.q4_0_dequant(bytes.fromhex(c["blocks_hex"]), c["n"])
    np.testing.assert_allclose(got, np.array(c["expect"], dtype=np.float32), atol=c["tol"], rtol=0)
    assert np.array_equal(got, np.array(c["expect"], dtype=np.float32))


def test_q4_0_interleaved_order():
    blk = bytes([0x00, 0x3C]) + bytes([(0xA << 4) | 0x3] + [0x88] * 15)
    w = ref.q4_0_dequant(blk, 32)
    assert w[0] == 3 - 8 and w[1] == 0xA - 8 and np.all(w[2:] == 0)


def test_q4_0_dot_nan_scale(kats):
    c = kats["q4_0_dot_nan"]
    assert c["half"] == 0xFE66
    got = ref.q_dot(ref.GGML_Q4_0, bytes.fromhex(c["blocks_hex"]), np.array(c["x"], dtype=np.float32))
    assert math.isnan(got)


def test_q8_0_dequant_signed():
    qs = np.arange(-16, 16, dtype=np.int8).view(np.uint8)
    blk = bytes([0x00, 0x40]) + qs.tobytes()  # d = 2.0
    assert np.array_equal(ref.q8_0_dequant(blk, 32), np.arange(-16, 16, dtype=np.float32) * 2)


def test_kernels_formulas(kats):
    k = kats["kernels"]
    x = np.array(k["rmsnorm"]["x"], dtype=np.float32)
    w = np.array(k["rmsnorm"]["w"], dtype=np.float32)
    a = x.copy()
    ref.rmsnorm_inplace(a, w, k["rmsnorm"]["eps"])
    inv = 1.0 / math.sqrt(float(np.float32(np.sum(x.astype(np.float64) ** 2) / 16 + 1e-5)))
    np.testing.assert_allclose(a, x * inv * w, rtol=1e-5, atol=k["rmsnorm"]["tol"])

    s = np.array(k["silu"]["x"], dtype=np.float32)
    ref.silu_inplace(s)
    np.testing.assert_allclose(s, k["silu"]["expect"], atol=k["silu"]["tol"])

    sm = np.array(k["softmax"]["x"], dtype=np.float32)
    ref.softmax_inplace(sm)
    np.testing.assert_allclose(sm, k["softmax"]["expect"], atol=k["softmax"]["tol"])

    s2 = np.array(k["softmax_sum"]["x"], dtype=np.float32)
    ref.softmax_inplace(s2)
    assert abs(float(s2.sum()) - 1.0) < k["softmax_sum"]["tol"]

    r = k["rope_invertible"]
    v = np.array(r["x"], dtype=np.float32)
    c, sn = np.array(r["cos"], dtype=np.float32), np.array(r["sin"], dtype=np.float32)
    ref.rope_inplace(v, c, sn, r["head_dim"])
    ref.rope_inplace(v, c, -sn, r["head_dim"])
    np.testing.assert_allclose(v, r["x"], atol=r["tol"])

    g = k["sgemm"]
    np.testing.assert_allclose(ref.sgemm(np.array(g["A"]), np.array(g["B"])), g["expect"], atol=g["tol"])
    g = k["sgemv"]
    np.testing.assert_allclose(ref.sgemv(np.array(g["A"], dtype=np.float32), np.array(g["x"], dtype=np.float32)),
                               g["expect"], rtol=1e-6, atol=g["tol"])


def test_sampler_kats(kats):
    for c in kats["sampler"]:
        t, k, p, rp, seed = c["config"]
        cfg = ref.SamplerConfig(t, k, p, rp, seed if seed else 12345)
        logits = np.array(c["logits"], dtype=np.float32)
        tok = ref.sample(logits.copy(), c["history"], cfg)
        assert tok in c["expect"], c["name"]
        if "first" in c:
            assert tok == c["first"]


def test_rope_table_matches_definition():
    cs, sn = ref.rope_tables(8, 10000.0, 4)
    for p in range(4):
        for i in range(4):
            f = np.float32(math.pow(10000.0, -2.0 * i / 8))
            a = np.float32(np.float32(p) * f)
            assert cs[p, 2 * i] == cs[p, 2 * i + 1] == np.float32(math.cos(float(a)))
            assert sn[p, 2 * i] == np.float32(math.sin(float(a)))


def test_model_ref_smoke():
    from auratensor_b200 import synth
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=1)
    cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                          shape.rope_theta, shape.eps, shape.vocab)
    m = ref.LlamaModelRef(cfg, t)
    logits = m.forward_step(5, 0)
    assert logits.shape == (shape.vocab,) and np.all(np.isfinite(logits))
    assert m.kv.size == 1
    with pytest.raises(RuntimeError):
        m.kv.append(0, shape.ctx, np.zeros(64, np.float32), np.zeros(64, np.float32))


def test_missing_output_weight_gives_zero_logits():
    # inference/Weights.java:131-135: an absent tensor becomes zeros
    from auratensor_b200 import synth
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=2)
    del t["output.weight"]
    cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                          shape.rope_theta, shape.eps, shape.vocab)
    assert np.all(ref.LlamaModelRef(cfg, t).forward_step(1, 0) == 0)


@pytest.mark.parametrize("which", ["reference_layout", "llama_cpp_layout", "q8_0_kv"])
def test_c_restatement_matches_numpy_oracle(which):
    """The C restatement (CPU baseline) and the numpy oracle agree on a tiny
    model, in the reference's byte layout, in llama.cpp's (split-halves
    Q4_0, [out][in] attention, Q6_K embedding and output) and with the Q8_0
    KV-cache rounding."""
    from auratensor_b200 import synth
    from oracle.cref import RefDecoder
    shape = synth.TINY_LLAMACPP if which == "llama_cpp_layout" else synth.TINY
    kv_type = ref.GGML_Q8_0 if which == "q8_0_kv" else 0
    t = synth.generate_numpy(shape, seed=31)
    cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                          shape.rope_theta, shape.eps, shape.vocab)
    a = ref.LlamaModelRef(cfg, t, layout=shape.layout, kv_type=kv_type)
    b = RefDecoder(shape, threads=2, kv_type=kv_type)
    for name, tt in t.items():
        b.set_tensor(name, tt["type"], tt["data"], int(np.prod(tt["dims"])))
    for pos, tok in enumerate([3, 99, 500, 7, 7]):
        la = a.forward_step(tok, pos)
        lb = b.forward_step(tok, pos)
        assert np.max(np.abs(la - lb)) <= 1e-5 * float(la.max() - la.min())


def test_q6_k_dequant_golden(kats):
    """The oracle's Q6_K decode against quant/Q6_KTest.java's cases."""
    for c in kats["q6_k_dequant"]:
        got = ref.q6_k_dequant(bytes.fromhex(c["block_hex"]), 256)
        want = np.array(c["expect"], dtype=np.float32)
        assert np.array_equal(got, want), c["name"]


def test_q4_0_split_halves_order():
    """llama.cpp's nibble order: element k = low nibble of byte k, k + 16 = high nibble."""
    blk = bytes([0x00, 0x3C]) + bytes(((k + 1) % 16) | ((15 - k) << 4) for k in range(16))  # d = 1.0
    w = ref.q4_0_dequant_split(blk, 32)
    assert [int(v) + 8 for v in w[:16]] == [(k + 1) % 16 for k in range(16)]
    assert [int(v) + 8 for v in w[16:]] == [15 - k for k in range(16)]


def test_llama_cpp_layout_is_the_same_model():
    """A llama.cpp-layout export of the same weights (split-halves nibbles,
    [out][in] attention) decodes to the reference-layout model's logits."""
    import dataclasses

    from auratensor_b200 import synth
    base = dataclasses.replace(synth.TINY, layout=synth.LAYOUT_LLAMA_CPP)
    t = synth.generate_numpy(base, seed=32)
    # the reference layout: interleaved nibbles, attention bytes [in][out]
    t_ref = {}
    for name, v in t.items():
        dims, data, tt = v["dims"], v["data"], v["type"]
        if tt == ref.GGML_Q4_0 and name.endswith(ref.ATTN_PROJ):
            # [out][in] -> the reference's [in][out] reading, as exact floats
            w = ref.q4_0_dequant_split(data, int(np.prod(dims))).reshape(dims)
            data, dims, tt = np.ascontiguousarray(w.T).view(np.uint8).reshape(-1), dims[::-1], ref.GGML_F32
        elif tt == ref.GGML_Q4_0:
            # split-halves -> interleaved nibbles: the same quants and scales
            raw = np.frombuffer(memoryview(data), dtype=np.uint8).reshape(-1, 18)
            q = np.concatenate([raw[:, 2:] & 0xF, raw[:, 2:] >> 4], axis=1)  # elements 0..31
            out = raw.copy()
            out[:, 2:] = q[:, 0::2] | (q[:, 1::2] << 4)
            data = out.reshape(-1)
        t_ref[name] = {"type": tt, "dims": dims, "data": data}
    cfg = ref.LlamaConfig(base.ctx, base.dim, base.n_layers, base.n_heads, base.n_kv_heads, base.ffn,
                          base.rope_theta, base.eps, base.vocab)
    a = ref.LlamaModelRef(cfg, t, layout=synth.LAYOUT_LLAMA_CPP)
    b = ref.LlamaModelRef(cfg, t_ref)
    for pos, tok in enumerate([3, 99, 500]):
        la, lb = a.forward_step(tok, pos), b.forward_step(tok, pos)
        assert np.max(np.abs(la - lb)) <= 1e-5 * float(lb.max() - lb.min())


def test_kv_q8_rounding():
    """The Q8_0 KV rounding: zero blocks stay zero, the block maximum is kept
    to fp16 precision, every value is within half a step d / 2 (plus the
    fp16 rounding of d), ties round away from zero."""
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(32 * 50) * rng.choice([1e-3, 1.0, 40.0], 32 * 50)).astype(np.float32)
    x[:32] = 0.0
    y = ref.kv_q8_roundtrip(x)
    assert np.all(y[:32] == 0)
    xb, yb = x.reshape(-1, 32), y.reshape(-1, 32)
    d = np.max(np.abs(xb), axis=1) / 127.0
    assert np.all(np.abs(xb - yb) <= d[:, None] * (0.5 + 127 * 2.0 ** -11) + 1e-30)
    # 0.5 * d lands exactly half way: rounds away from zero
    t = np.zeros(32, dtype=np.float32)
    t[0], t[1], t[2] = 127.0, 0.5, -0.5
    assert ref.kv_q8_roundtrip(t)[1:3].tolist() == [1.0, -1.0]
