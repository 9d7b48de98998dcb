"""llama.cpp-layout GGUF exports on the device path: split-halves Q4_0
nibbles, attention weights stored [out][in], Q6_K token embedding and
lm_head. The reference reads only its own layout (interleaved nibbles,
quant/Q4_0.java:21-22; attention [in][out], inference/LlamaModel.java:326-369)
and dequantizes Q6_K at load (quant/Q6_K.java, inference/Weights.java:204-216);
the oracle variant restates those readings for the llama.cpp layout
(oracle/ref.py: q4_0_dequant_split, q6_k_dequant, LlamaModelRef(layout=...)).

Rules: codecs bit-exact; GEMVs within 2e-5 x sum |w x| per output; decode
logits within 1e-3 x (max - min of the oracle's logits); the batched prompt
path within 2e-2 of the range.
"""
import dataclasses
import os

import numpy as np
import pytest
import torch

from auratensor_b200 import _lib, synth
from auratensor_b200.inference import LlamaConfig, LlamaModel
from auratensor_b200.quant import ORIENT_N, ORIENT_T, Q6_K, QMatrix
from oracle import ref

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3
GEMV_TOL = 2e-5
LCPP = synth.LAYOUT_LLAMA_CPP


def oracle_cfg(s):
    return ref.LlamaConfig(s.ctx, s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.ffn, s.rope_theta, s.eps, s.vocab)


def test_q6_k_codec_bit_exact(kats, cuda):
    rng = np.random.default_rng(5)
    blocks = synth.quantize_q6_k((rng.standard_normal(256 * 64) * 0.02).astype(np.float32))
    blocks = np.concatenate([blocks] + [np.frombuffer(bytes.fromhex(c["block_hex"]), dtype=np.uint8)
                                        for c in kats["q6_k_dequant"]])
    n = blocks.size // 210 * 256
    got = Q6_K.dequantToFloat(torch.from_numpy(blocks).to(cuda), None, n).cpu().numpy()
    want = ref.q6_k_dequant(blocks.tobytes(), n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("orient", [ORIENT_N, ORIENT_T])
def test_split_halves_matrix_is_stored_interleaved(orient, cuda):
    rows, cols = 96, 256
    rng = np.random.default_rng(6)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    split = synth.quantize_q4_0(w, split=True)
    m = QMatrix(ref.GGML_Q4_0, orient, rows, cols, torch.from_numpy(split).to(cuda), layout=synth.LAYOUT_Q4_SPLIT_HALVES)
    exported = m.export_blocks().cpu().numpy()
    assert np.array_equal(exported, synth.quantize_q4_0(w, split=False))
    W = ref.q4_0_dequant_split(split.tobytes(), rows * cols).reshape(rows, cols).astype(np.float64)
    n_in = cols if orient == ORIENT_N else rows
    x = rng.standard_normal((2, n_in)).astype(np.float32)
    y = m.gemv(torch.from_numpy(x).to(cuda)).cpu().numpy()
    Wo = W if orient == ORIENT_N else W.T
    want = x.astype(np.float64) @ Wo.T
    bound = GEMV_TOL * (np.abs(x).astype(np.float64) @ np.abs(Wo.T)) + 1e-30
    assert np.all(np.abs(y - want) <= bound)


@pytest.mark.parametrize("rows,cols,batch", [(1000, 256, 1), (1000, 256, 8), (32000, 4096, 2), (32000, 4096, 8),
                                             (128256, 4096, 1)])
def test_q6_k_gemv(rows, cols, batch, cuda):
    g = torch.Generator(device=cuda).manual_seed(rows + batch)
    blocks = synth.generate_torch_tensor((rows, cols), synth.Q6_K, g, cuda)
    m = QMatrix(synth.Q6_K, ORIENT_N, rows, cols, blocks)
    assert torch.equal(m.export_blocks(), blocks)
    W = ref.q6_k_dequant(blocks.cpu().numpy().tobytes(), rows * cols).reshape(rows, cols).astype(np.float64)
    x = torch.randn((batch, cols), device=cuda)
    y = m.gemv(x).cpu().numpy()
    xd = x.cpu().numpy().astype(np.float64)
    want = xd @ W.T
    bound = GEMV_TOL * (np.abs(xd) @ np.abs(W.T)) + 1e-30
    assert np.all(np.abs(y - want) <= bound)


def teacher_forced(gpu, orc, toks):
    worst = 0.0
    for pos, tok in enumerate(toks):
        lr = orc.forward_step(int(tok), pos)
        lg = gpu.forwardStep(int(tok), pos).copy()
        rng_ = float(lr.max() - lr.min())
        err = float(np.max(np.abs(lg - lr)))
        assert err <= REL_TOL * rng_, (pos, err, rng_)
        worst = max(worst, err / rng_)
    return worst


def test_llama_cpp_tiny_teacher_forced(cuda):
    shape = synth.TINY_LLAMACPP
    t = synth.generate_numpy(shape, seed=51)
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t, layout=LCPP)
    orc = ref.LlamaModelRef(oracle_cfg(shape), t, layout=LCPP)
    teacher_forced(gpu, orc, synth.prompt_ids(shape, 51, shape.ctx).tolist())
    kv = gpu.kvCache()
    for layer in range(shape.n_layers):
        for h in range(shape.n_kv_heads):
            for p in (0, 17, shape.ctx - 1):
                k, v = kv.read(layer, h, p)
                np.testing.assert_allclose(k, orc.kv.k[layer, h, p], rtol=1e-4, atol=1e-5)
                np.testing.assert_allclose(v, orc.kv.v[layer, h, p], rtol=1e-4, atol=1e-5)


def test_llama_cpp_batched_decode(cuda):
    """Slots at different positions through the [out][in] QKV and its RoPE/KV kernel."""
    shape = synth.TINY_LLAMACPP
    t = synth.generate_numpy(shape, seed=52)
    B = 4
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t, max_batch=B, layout=LCPP)
    orcs = [ref.LlamaModelRef(oracle_cfg(shape), t, layout=LCPP) for _ in range(B)]
    rng = np.random.default_rng(52)
    pos = [0] * B
    for step in range(12):
        if step == 5:  # restart slot 2 from position 0
            gpu.kvCache(2).reset()
            orcs[2] = ref.LlamaModelRef(oracle_cfg(shape), t, layout=LCPP)
            pos[2] = 0
        toks = [int(v) for v in rng.integers(0, shape.vocab, size=B)]
        lg = gpu.forwardBatch(toks, pos).copy()
        for b in range(B):
            lr = orcs[b].forward_step(toks[b], pos[b])
            assert np.max(np.abs(lg[b] - lr)) <= REL_TOL * float(lr.max() - lr.min()), (step, b)
        pos = [p + 1 for p in pos]


def test_llama_cpp_prompt_path(cuda):
    # 600 tokens: a 512-token chunk of the batched prompt path and a short one
    shape = dataclasses.replace(synth.TINY_LLAMACPP, ctx=640)
    t = synth.generate_numpy(shape, seed=53)
    n = 600
    prompt = synth.prompt_ids(shape, 53, n + 3).tolist()
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t, layout=LCPP)
    orc = ref.LlamaModelRef(oracle_cfg(shape), t, layout=LCPP)
    gpu.forwardPrompt(prompt[:n])
    for pos in range(n):
        orc.forward_step(prompt[pos], pos)
    for i in range(3):
        lg = gpu.forwardStep(prompt[n + i], n + i).copy()
        lr = orc.forward_step(prompt[n + i], n + i)
        assert np.max(np.abs(lg - lr)) <= 2e-2 * float(lr.max() - lr.min())


def test_llama_cpp_gguf_load(tmp_path, cuda):
    shape = synth.TINY_LLAMACPP
    t = synth.generate_numpy(shape, seed=54)
    path = str(tmp_path / "tiny-llamacpp.gguf")
    synth.write_gguf(shape, t, path)
    a = LlamaModel(LlamaConfig.fromShape(shape), t, layout=LCPP)
    b = LlamaModel.fromGguf(path, layout=LCPP)
    first = None
    for pos, tok in enumerate([3, 17, 999, 0]):
        la = a.forwardStep(tok, pos).copy()
        assert np.array_equal(la, b.forwardStep(tok, pos).copy())
        first = la if first is None else first
    # read in the reference's layout, the same file decodes differently
    c = LlamaModel.fromGguf(path)
    assert not np.array_equal(c.forwardStep(3, 0).copy(), first)


def test_llama_cpp_8b_dims(cuda):
    """Llama-3-8B dims in the llama.cpp layout (1 layer; the lm_head is a
    128256 x 4096 Q6_K matrix) against the C oracle."""
    from oracle.cref import RefDecoder
    shape = dataclasses.replace(synth.LLAMA3_8B, n_layers=1, ctx=48, layout=LCPP, emb_type=synth.Q6_K)
    g = torch.Generator(device="cuda").manual_seed(55)
    gpu = LlamaModel(LlamaConfig.fromShape(shape), None, layout=LCPP)
    orc = RefDecoder(shape, threads=os.cpu_count() or 1)
    for name, dims, tt in shape.tensor_dims():
        data = synth.generate_torch_tensor(dims, tt, g, "cuda", layout=LCPP)
        gpu.setTensor(name, tt, data)
        orc.set_tensor(name, tt, data.cpu().numpy(), int(np.prod(dims)))
        del data
    gpu.finalize()
    teacher_forced(gpu, orc, np.random.default_rng(56).integers(0, shape.vocab, 24).tolist())
    orc.close()


def test_q6_k_only_for_embedding_and_output(cuda):
    shape = synth.TINY
    m = LlamaModel(LlamaConfig.fromShape(shape), None)
    blocks = synth.quantize_q6_k(np.zeros(256 * 256, dtype=np.float32))
    with pytest.raises(_lib.UnsupportedOperationException):
        m.setTensor("blk.0.ffn_gate.weight", synth.Q6_K, blocks)
