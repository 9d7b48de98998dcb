"""The persistent decode step (one launch per token: every layer, the lm_head
and the greedy argmax in one kernel with one CTA per SM; opt-in with
AT_DECODE_STEP=1 at load) against the oracle and against the per-kernel step
graph (the default).

Rules as for the other decode tests: logits within 1e-3 x (max - min of the
oracle's logits); greedy tokens equal except where the oracle's top-2 gap is
below that. Between the two device paths (both FP32, different summation
orders) the same bound applies.
"""
import os

import numpy as np
import pytest

from auratensor_b200 import synth
from auratensor_b200.inference import LlamaConfig, LlamaModel
from oracle import ref

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3


def oracle_cfg(s):
    return ref.LlamaConfig(s.ctx, s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.ffn, s.rope_theta, s.eps, s.vocab)


def graph_model(shape, t):
    return LlamaModel(LlamaConfig.fromShape(shape), t)


def persistent_model(shape, t):
    os.environ["AT_DECODE_STEP"] = "1"
    try:
        return LlamaModel(LlamaConfig.fromShape(shape), t)
    finally:
        del os.environ["AT_DECODE_STEP"]


@pytest.mark.parametrize("shape", [synth.TINY, synth.TINY_Q8], ids=["q4_0", "q8_0"])
def test_persistent_step_matches_oracle_and_graph(shape, cuda):
    t = synth.generate_numpy(shape, seed=41)
    ps = persistent_model(shape, t)
    gr = graph_model(shape, t)
    assert ps.persistentStep() and not gr.persistentStep()
    orc = ref.LlamaModelRef(oracle_cfg(shape), t)
    toks = synth.prompt_ids(shape, 41, shape.ctx).tolist()
    for pos in range(shape.ctx):
        lr = orc.forward_step(toks[pos], pos)
        a = ps.forwardStep(toks[pos], pos).copy()
        b = gr.forwardStep(toks[pos], pos).copy()
        rng_ = float(lr.max() - lr.min())
        assert np.max(np.abs(a - lr)) <= REL_TOL * rng_, pos
        assert np.max(np.abs(a - b)) <= REL_TOL * rng_, pos
        assert ps.argmax(1)[0] == int(np.argmax(a))
    kv_p, kv_g = ps.kvCache(), gr.kvCache()
    for layer in range(shape.n_layers):
        for h in range(shape.n_kv_heads):
            for p in (0, 7, shape.ctx - 1):
                k1, v1 = kv_p.read(layer, h, p)
                k2, v2 = kv_g.read(layer, h, p)
                np.testing.assert_allclose(k1, k2, rtol=1e-4, atol=1e-5)
                np.testing.assert_allclose(v1, v2, rtol=1e-4, atol=1e-5)


def test_persistent_greedy_loop_matches_graph_loop(cuda):
    """at_model_generate: the argmax and the token/position advance happen
    inside the persistent kernel; the sequence equals the graph path's."""
    shape = synth.LLAMA32_1B
    t = synth.generate_numpy(shape, seed=42)
    ps = persistent_model(shape, t)
    gr = graph_model(shape, t)
    prompt = synth.prompt_ids(shape, 42, 8).tolist()
    ps.forwardPrompt(prompt)
    gr.forwardPrompt(prompt)
    a = ps.generate(prompt[-1], len(prompt), 48)
    b = gr.generate(prompt[-1], len(prompt), 48)
    assert ps.kvCache().size() == len(prompt) + 48
    # equal unless a near tie flips one greedy token (then the rest diverges)
    same = int(np.argmax(a != b)) if np.any(a != b) else len(a)
    assert same >= 16, (a.tolist(), b.tolist())


def test_persistent_step_early_positions_many_ctas(cuda):
    """Positions 0..40 on a model with one KV head group per 32 attention CTAs:
    most CTAs of a head have no positions yet and contribute empty partials."""
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=43)
    ps = persistent_model(shape, t)
    assert ps.persistentStep()
    orc = ref.LlamaModelRef(oracle_cfg(shape), t)
    for pos in range(40):
        lr = orc.forward_step(pos % shape.vocab, pos)
        a = ps.forwardStep(pos % shape.vocab, pos)
        assert np.max(np.abs(a - lr)) <= REL_TOL * float(lr.max() - lr.min()), pos


@pytest.mark.parametrize("base,layers,ctx,check", [
    (synth.LLAMA3_8B, 2, 1100, (0, 1, 63, 511, 1023, 1024, 1099)),   # head_dim 128, GQA 4
    (synth.LLAMA3_70B, 1, 40, tuple(range(0, 40, 3))),             # dim 8192, GQA 8
], ids=["llama3-8b-2l", "llama3-70b-1l"])
def test_persistent_step_benchmark_shapes(base, layers, ctx, check, cuda):
    """The persistent kernel at true benchmark dims against the C oracle."""
    import dataclasses

    import torch

    from oracle.cref import RefDecoder
    shape = dataclasses.replace(base, n_layers=layers, ctx=ctx)
    g = torch.Generator(device="cuda").manual_seed(90)
    os.environ["AT_DECODE_STEP"] = "1"
    try:
        gpu = LlamaModel(LlamaConfig.fromShape(shape), None)
        orc = RefDecoder(shape, threads=os.cpu_count() or 1)
        for name, dims, t in shape.tensor_dims():
            data = synth.generate_torch_tensor(dims, t, g, "cuda")
            gpu.setTensor(name, t, data)
            orc.set_tensor(name, t, data.cpu().numpy(), int(np.prod(dims)))
            del data
        gpu.finalize()
    finally:
        del os.environ["AT_DECODE_STEP"]
    assert gpu.persistentStep()
    toks = np.random.default_rng(91).integers(0, shape.vocab, ctx)
    for pos in range(ctx):
        if pos in check:
            lr = orc.forward_step(int(toks[pos]), pos)
            lg = gpu.forwardStep(int(toks[pos]), pos)
            assert np.max(np.abs(lg - lr)) <= REL_TOL * float(lr.max() - lr.min()), pos
        else:
            orc.forward_layers(int(toks[pos]), pos)
            gpu.forwardStepDevice(int(toks[pos]), pos)
    gpu.close()
    orc.close()
