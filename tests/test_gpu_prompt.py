"""Batched forwardPrompt (tensor-core GEMMs, bf16 operands) against the
oracle's token-by-token forwardStep.

The prompt path's rule: KV-cache contents and the following decode logits
within 2e-2 of the oracle's range (per layer and head for the cache). The
prompt path runs chunks of 512 tokens (the GEMMs' two 256-token tiles);
prompts of 7, 130 and 300 tokens are one chunk (one or two token tiles),
600 tokens a chunk boundary, 1100 tokens two whole chunks and a short one.
"""
import dataclasses

import numpy as np
import pytest

from auratensor_b200 import synth
from auratensor_b200.inference import LlamaConfig, LlamaModel
from oracle import ref

pytestmark = pytest.mark.gpu
PROMPT_TOL = 2e-2


def oracle_cfg(s):
    return ref.LlamaConfig(s.ctx, s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.ffn, s.rope_theta, s.eps, s.vocab)


@pytest.mark.parametrize("base", [synth.TINY, synth.TINY_Q8], ids=["q4_0", "q8_0"])
@pytest.mark.parametrize("n", [7, 130, 300, 600, 1100])
def test_batched_prompt_matches_oracle(base, n, cuda):
    shape = dataclasses.replace(base, ctx=1200)
    t = synth.generate_numpy(shape, seed=31)
    prompt = synth.prompt_ids(shape, 31, n + 4).tolist()
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t)
    orc = ref.LlamaModelRef(oracle_cfg(shape), t)
    gpu.forwardPrompt(prompt[:n])
    for pos in range(n):
        orc.forward_step(prompt[pos], pos)
    kv = gpu.kvCache()
    assert kv.size() == n
    for layer in range(shape.n_layers):
        for h in range(shape.n_kv_heads):
            kr, vr = orc.kv.k[layer, h, :n], orc.kv.v[layer, h, :n]
            k = np.stack([kv.read(layer, h, p)[0] for p in range(n)])
            v = np.stack([kv.read(layer, h, p)[1] for p in range(n)])
            assert np.max(np.abs(k - kr)) <= PROMPT_TOL * float(kr.max() - kr.min())
            assert np.max(np.abs(v - vr)) <= PROMPT_TOL * float(vr.max() - vr.min())
    for i in range(4):
        lg = gpu.forwardStep(prompt[n + i], n + i).copy()
        lr = orc.forward_step(prompt[n + i], n + i)
        assert np.max(np.abs(lg - lr)) <= PROMPT_TOL * float(lr.max() - lr.min())


def test_batched_prompt_is_deterministic(cuda):
    shape = dataclasses.replace(synth.TINY, ctx=512)
    t = synth.generate_numpy(shape, seed=32)
    prompt = synth.prompt_ids(shape, 32, 200).tolist()
    a, b = LlamaModel(LlamaConfig.fromShape(shape), t), LlamaModel(LlamaConfig.fromShape(shape), t)
    a.forwardPrompt(prompt)
    b.forwardPrompt(prompt)
    for p in (0, 127, 128, 199):
        ka, va = a.kvCache().read(1, 1, p)
        kb, vb = b.kvCache().read(1, 1, p)
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    assert np.array_equal(a.forwardStep(3, 200), b.forwardStep(3, 200))
