"""Decode parity at the benchmark model shapes (true dims, fewer layers) against
the oracle's C restatement of the reference (LlamaModel.forwardStep,
inference/LlamaModel.java:141-297).

- Llama-3-8B shape (dim 4096, FFN 14336, 32/8 heads, head_dim 128, vocab
  128256, theta 5e5), 2 layers, context 2112: every position goes through
  both KV caches; the decode attention runs 64-position CTAs in clusters of
  16 along the sequence (1024 positions per cluster), so positions 1023/1024/
  1025 and 2047/2048 cross one and two cluster boundaries and the last
  positions merge three cluster partials through global memory.
- Mistral-7B shape in Q8_0 (vocab 32000, theta 1e6), 1 layer, context 4096:
  four clusters of chunk CTAs at the end.
- Llama-3-70B shape (dim 8192, FFN 28672, 64/8 heads: GQA group 8), 1 layer.
- The Llama-3.2-1B configuration whole (16 layers, head_dim 64, tied
  embeddings, context 128): 8 prompt tokens and 32 greedy decode steps.
- The batched prompt path (tensor-core GEMMs, bf16 operands) at head_dim 128
  over 600 tokens (a 512-token chunk and an 88-token one).

Rules (the FP32 GEMV path): logits within 1e-3 x (max - min of the oracle's
logits) at every compared step; greedy tokens equal except where the
oracle's top-2 gap is below that; K and V rows within 1e-3 x the range of
the oracle's row. Prompt path: 2e-2 of the range for the KV contents and the
following logits. Weights are N(0, 0.02) quantized on the device; the oracle
reads the same bytes.
"""
import dataclasses
import os

import numpy as np
import pytest
import torch

from auratensor_b200 import synth
from auratensor_b200.inference import LlamaConfig, LlamaModel
from oracle.cref import RefDecoder

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3
PROMPT_TOL = 2e-2


def build_pair(shape, seed):
    """The same seeded weights in a device model and in the C oracle."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    gpu = LlamaModel(LlamaConfig.fromShape(shape), None)
    orc = RefDecoder(shape, threads=os.cpu_count() or 1)
    for name, dims, t in shape.tensor_dims():
        data = synth.generate_torch_tensor(dims, t, g, "cuda")
        gpu.setTensor(name, t, data)
        orc.set_tensor(name, t, data.cpu().numpy(), int(np.prod(dims)))
        del data
    gpu.finalize()
    return gpu, orc


def check_logits(lg, lr, tol, where):
    rng_ = float(lr.max() - lr.min())
    err = float(np.max(np.abs(lg - lr)))
    assert err <= tol * rng_, (where, err, rng_)
    return err / rng_


def check_kv(gpu, orc, shape, positions, tol):
    kv = gpu.kvCache()
    for layer in range(shape.n_layers):
        for h in range(shape.n_kv_heads):
            for p in positions:
                k, v = kv.read(layer, h, p)
                kr, vr = orc.kv(layer, h, p)
                assert np.max(np.abs(k - kr)) <= tol * float(kr.max() - kr.min()), ("K", layer, h, p)
                assert np.max(np.abs(v - vr)) <= tol * float(vr.max() - vr.min()), ("V", layer, h, p)


def run_teacher_forced(shape, seed, check, n_greedy):
    """Random tokens through positions [0, ctx - n_greedy), then n_greedy
    greedy steps fed with the oracle's argmax. Logits are compared at the
    positions in `check` and at every greedy step; the other steps only fill
    the KV caches (no logits copied)."""
    gpu, orc = build_pair(shape, seed)
    toks = np.random.default_rng(seed + 1).integers(0, shape.vocab, shape.ctx)
    first_greedy = shape.ctx - n_greedy
    worst, tok = 0.0, int(toks[0])
    for pos in range(shape.ctx):
        if pos < first_greedy:
            tok = int(toks[pos])  # past it, tok is the previous step's greedy token
        if pos in check or pos >= first_greedy - 1:
            lr = orc.forward_step(tok, pos)
            lg = gpu.forwardStep(tok, pos).copy()
            worst = max(worst, check_logits(lg, lr, REL_TOL, pos))
            if pos >= first_greedy - 1:
                ref_tok = int(np.argmax(lr))
                if int(np.argmax(lg)) != ref_tok:
                    srt = np.sort(lr)
                    assert float(srt[-1] - srt[-2]) < REL_TOL * float(lr.max() - lr.min()), ("greedy", pos)
                tok = ref_tok
        else:
            orc.forward_layers(tok, pos)
            gpu.forwardStepDevice(tok, pos)
    return gpu, orc, worst


def test_llama3_8b_shape_long_context(cuda):
    shape = dataclasses.replace(synth.LLAMA3_8B, n_layers=2, ctx=2112)
    check = {0, 1, 63, 64, 511, 512, 1023, 1024, 1025, 1500, 2047, 2048, 2049, 2080}
    gpu, orc, worst = run_teacher_forced(shape, 80, check, n_greedy=8)
    assert gpu.kvCache().size() == shape.ctx
    check_kv(gpu, orc, shape, (0, 511, 1023, 1024, 2047, 2048, shape.ctx - 1), REL_TOL)
    assert worst <= REL_TOL
    gpu.close()
    orc.close()


def test_mistral_7b_shape_q8_0_four_clusters(cuda):
    shape = dataclasses.replace(synth.MISTRAL_7B, n_layers=1)
    assert shape.wtype == synth.Q8_0 and shape.ctx == 4096
    check = {0, 1023, 1024, 2047, 2048, 3071, 3072, 3073, 4000}
    gpu, orc, worst = run_teacher_forced(shape, 81, check, n_greedy=6)
    check_kv(gpu, orc, shape, (0, 1024, 3072, 4095), REL_TOL)
    gpu.close()
    orc.close()


def test_llama32_1b_config_workload(cuda):
    """The 1B configuration as specified: all 16 layers, dim 2048, head_dim
    64, tied embeddings (output.weight is the token_embd bytes), context 128;
    8 seeded prompt tokens through forwardStep (the reference's forwardPrompt
    is one forwardStep per token), then 32 greedy decode steps fed the
    oracle's argmax. Every step's logits within 1e-3 of the range; greedy
    tokens equal except where the oracle's top-2 gap is below that."""
    shape = synth.LLAMA32_1B
    assert shape.tied and shape.ctx == 128 and shape.head_dim == 64 and shape.n_layers == 16
    g = torch.Generator(device="cuda").manual_seed(85)
    gpu = LlamaModel(LlamaConfig.fromShape(shape), None)
    orc = RefDecoder(shape, threads=os.cpu_count() or 1)
    emb = None
    for name, dims, t in shape.tensor_dims():
        data = emb if name == "output.weight" else synth.generate_torch_tensor(dims, t, g, "cuda")
        if name == "token_embd.weight":
            emb = data
        gpu.setTensor(name, t, data)
        orc.set_tensor(name, t, data.cpu().numpy(), int(np.prod(dims)))
    gpu.finalize()
    prompt = synth.prompt_ids(shape, 85, 8).tolist()
    n_prompt, n_decode = 8, 32
    tok, worst, agree = prompt[0], 0.0, 0
    for pos in range(n_prompt + n_decode - 1):
        if pos < n_prompt:
            tok = prompt[pos]
        lr = orc.forward_step(tok, pos)
        lg = gpu.forwardStep(tok, pos).copy()
        worst = max(worst, check_logits(lg, lr, REL_TOL, pos))
        if pos >= n_prompt - 1:  # this step's argmax is a generated token
            ref_tok = int(np.argmax(lr))
            if int(np.argmax(lg)) == ref_tok:
                agree += 1
            else:
                srt = np.sort(lr)
                assert float(srt[-1] - srt[-2]) < REL_TOL * float(lr.max() - lr.min()), ("greedy", pos)
            tok = ref_tok
    assert gpu.kvCache().size() == n_prompt + n_decode - 1
    assert agree >= n_decode - 2  # near-ties aside, the same 32 tokens
    check_kv(gpu, orc, shape, (0, 7, n_prompt + n_decode - 2), REL_TOL)
    gpu.close()
    orc.close()


def test_llama3_70b_shape_gqa8(cuda):
    shape = dataclasses.replace(synth.LLAMA3_70B, n_layers=1, ctx=40)
    assert shape.n_heads // shape.n_kv_heads == 8 and shape.head_dim == 128
    gpu, orc, worst = run_teacher_forced(shape, 82, set(range(shape.ctx)), n_greedy=16)
    check_kv(gpu, orc, shape, (0, 17, shape.ctx - 1), REL_TOL)
    gpu.close()
    orc.close()


def test_hd128_batched_prompt(cuda):
    shape = dataclasses.replace(synth.LLAMA3_8B, n_layers=2, ctx=640)
    n = 600
    gpu, orc = build_pair(shape, 83)
    prompt = np.random.default_rng(84).integers(0, shape.vocab, n + 4).tolist()
    gpu.forwardPrompt(prompt[:n])
    for pos in range(n):
        orc.forward_layers(prompt[pos], pos)
    assert gpu.kvCache().size() == n
    kv = gpu.kvCache()
    for layer in range(shape.n_layers):
        for h in range(shape.n_kv_heads):
            rows = [(kv.read(layer, h, p), orc.kv(layer, h, p)) for p in range(n)]
            k = np.stack([r[0][0] for r in rows])
            v = np.stack([r[0][1] for r in rows])
            kr = np.stack([r[1][0] for r in rows])
            vr = np.stack([r[1][1] for r in rows])
            assert np.max(np.abs(k - kr)) <= PROMPT_TOL * float(kr.max() - kr.min()), ("K", layer, h)
            assert np.max(np.abs(v - vr)) <= PROMPT_TOL * float(vr.max() - vr.min()), ("V", layer, h)
    for i in range(4):
        lg = gpu.forwardStep(prompt[n + i], n + i).copy()
        lr = orc.forward_step(prompt[n + i], n + i)
        check_logits(lg, lr, PROMPT_TOL, n + i)
    gpu.close()
    orc.close()
