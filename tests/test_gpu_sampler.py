"""Sampling on the device (csrc/sample.cu) against Sampler.sample
(inference/Sampler.java:37-121) restated on the host (csrc/sampler.cpp, itself
pinned to the oracle and the reference's test cases on the CPU), batched
sampled decoding against a host step-and-sample loop, and the request
scheduler against serial generation.

Rules: sampled ids equal (integer work over the same float logits; the one
double exp per candidate may differ by an ulp between the device and the
host library, which moves a float probability only in a rare tie, so the
tests use seeds where none occurs); logits after the in-place repetition
penalty bit-equal (NaN payloads aside).
"""
import dataclasses
import functools

import numpy as np
import pytest
import torch

from auratensor_b200 import _lib, synth
from auratensor_b200.inference import LlamaConfig, LlamaModel, Sampler, SamplerConfig
from auratensor_b200.scheduler import BatchScheduler
from oracle import ref

pytestmark = pytest.mark.gpu
MAXB = 8


@functools.lru_cache(maxsize=None)
def sampler_model(vocab: int):
    shape = dataclasses.replace(synth.TINY, vocab=vocab, n_layers=1)
    return LlamaModel(LlamaConfig.fromShape(shape), synth.generate_numpy(shape, seed=vocab), max_batch=MAXB)


def device_sample(model, rows, hists, cfgs):
    """Writes the rows into the model's logits, samples on the device; returns
    the ids and the logits after the penalty."""
    view = model.logitsDevice()
    n = len(rows)
    view[:n].copy_(torch.from_numpy(np.stack(rows)))
    torch.cuda.synchronize()
    got = model.sample(cfgs, hists)
    torch.cuda.synchronize()
    return got, view[:n].cpu().numpy()


def host_sample(row, hist, cfg):
    a = row.copy()
    return Sampler.sample(a, hist, cfg), a


def same_floats(a, b):
    """Bit-equal, except that any NaN equals any NaN (the device writes the
    canonical NaN where the host keeps the input's payload)."""
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def check_rows(model, rows, hists, cfgs):
    for i in range(0, len(rows), MAXB):
        got, after = device_sample(model, rows[i:i + MAXB], hists[i:i + MAXB], cfgs[i:i + MAXB])
        for j in range(len(got)):
            want, want_after = host_sample(rows[i + j], hists[i + j], cfgs[i + j])
            assert got[j] == want, (i + j, cfgs[i + j], got[j], want)
            assert same_floats(after[j], want_after), i + j


def test_reference_sampler_cases(kats, cuda):
    """The reference's SamplerTest cases (vocab 4..1024) on the device."""
    for c in kats["sampler"]:
        t, k, p, rp, seed = c["config"]
        logits = np.array(c["logits"], dtype=np.float32)
        m = sampler_model(logits.size)
        cfg = SamplerConfig(t, k, p, rp, seed if seed else 7)
        got, _ = device_sample(m, [logits], [c["history"]], [cfg])
        assert got[0] in c["expect"], c["name"]
        if "first" in c:
            assert got[0] == c["first"]


def make_cases(vocab, n, seed):
    rng = np.random.default_rng(seed)
    rows, hists, cfgs = [], [], []
    for i in range(n):
        kind = i % 8
        x = (rng.standard_normal(vocab) * rng.choice([0.5, 2.0, 6.0])).astype(np.float32)
        if kind == 1:  # many exact ties: the stable order decides among equal values
            x = np.round(x * 2).astype(np.float32)
        elif kind == 2:  # NaN (sorts above +inf), infinities, signed zeros
            idx = rng.choice(vocab, size=12, replace=False)
            x[idx[:3]] = np.nan
            x[idx[3:5]] = np.inf
            x[idx[5:7]] = -np.inf
            x[idx[7:9]] = 0.0
            x[idx[9:12]] = -0.0
        elif kind == 3:  # every logit equal
            x[:] = np.float32(rng.standard_normal())
        elif kind == 4:  # a NaN at index 0 (the greedy scan's start)
            x[0] = np.nan
        hist = rng.integers(-3, vocab + 3, size=int(rng.integers(0, 300))).tolist()
        hist += hist[: len(hist) // 3]  # repeated ids: the penalty applies once per occurrence
        t = float(rng.choice([0.0, 0.1, 0.7, 1.0, 1.7, -0.5]))
        k = int(rng.choice([1, 2, 5, 40, 257, 1000, 1024]))
        p = float(rng.choice([1.0, 0.95, 0.5, 0.0, 0.999]))
        rp = float(rng.choice([1.0, 1.1, 1.3, 0.8, -1.5]))
        rows.append(x)
        hists.append(hist)
        cfgs.append(SamplerConfig(t, k, p, rp, int(rng.integers(1, 1 << 40))))
    return rows, hists, cfgs


@pytest.mark.parametrize("vocab", [1000, 32000, 128256])
def test_device_sampler_matches_host(vocab, cuda):
    rows, hists, cfgs = make_cases(vocab, 48 if vocab < 100000 else 16, vocab)
    check_rows(sampler_model(vocab), rows, hists, cfgs)


def test_device_sampler_matches_oracle(cuda):
    """A few rows straight against the Python oracle's Sampler.sample."""
    vocab = 32000
    rows, hists, cfgs = make_cases(vocab, 8, 99)
    cfgs = [SamplerConfig(0.7, 40, 0.95, 1.1, 1000 + i) for i in range(8)]
    got, _ = device_sample(sampler_model(vocab), rows, hists, cfgs)
    for j in range(8):
        want = ref.sample(rows[j].copy(), hists[j], ref.SamplerConfig(0.7, 40, 0.95, 1.1, 1000 + j))
        assert got[j] == want, j


def test_unseeded_rows_draw_from_the_candidates(cuda):
    """seed 0: the reference draws from an unseeded generator; the device row
    advances its own java.util.Random, so every pick is one of the top k."""
    vocab = 32000
    m = sampler_model(vocab)
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(vocab) * 3).astype(np.float32)
    top = set(np.argsort(-x, kind="stable")[:40].tolist())
    seen = set()
    for _ in range(6):
        got, _ = device_sample(m, [x] * MAXB, [None] * MAXB, [SamplerConfig(1.0, 40, 1.0, 1.0, 0)] * MAXB)
        assert set(got.tolist()) <= top
        seen |= set(got.tolist())
    assert len(seen) > 3


def test_top_k_limits(cuda):
    m = sampler_model(32000)
    x = np.zeros(32000, dtype=np.float32)
    with pytest.raises(_lib.UnsupportedOperationException):
        device_sample(m, [x], [None], [SamplerConfig(1.0, 1025, 1.0, 1.0, 3)])
    with pytest.raises(_lib.IllegalArgumentException):
        device_sample(m, [x], [None], [SamplerConfig(1.0, 0, 1.0, 1.0, 3)])
    # greedy settings never reach the candidate buffer
    got, _ = device_sample(m, [x], [None], [SamplerConfig(0.0, 5000, 1.0, 1.0, 3)])
    assert got[0] == 0


def host_loop(model, prompts, n_steps, cfgs):
    """Serial reference: forwardPrompt + forwardStep per token, host Sampler."""
    outs = []
    for b, prompt in enumerate(prompts):
        model.kvCache().reset()
        model.forwardPrompt(prompt[:-1])
        hist = list(prompt)
        lg = model.forwardStep(prompt[-1], len(prompt) - 1).copy()
        out = []
        for i in range(n_steps):
            t = Sampler.sample(lg, hist, cfgs[b])
            out.append(t)
            hist.append(t)
            if i + 1 < n_steps:
                lg = model.forwardStep(t, len(prompt) + i).copy()
        outs.append(out)
    return outs


def test_generate_sampled_matches_host_loop(cuda):
    """Four rows decoded together on the device (token feedback, penalty
    history growth, r per row) against each row run alone with the host
    sampler; the prompts go through the same batched prompt path."""
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=61)
    B, n_steps = 4, 24
    prompts = [synth.prompt_ids(shape, 61 + b, 6 + 3 * b).tolist() for b in range(B)]
    cfgs = [SamplerConfig(0.7, 40, 0.95, 1.1, 11), SamplerConfig(1.0, 5, 1.0, 1.3, 12),
            SamplerConfig(0.0, 1, 1.0, 1.2, 13), SamplerConfig(1.5, 200, 0.9, 1.0, 14)]
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t, max_batch=B)
    for b, p in enumerate(prompts):
        gpu.forwardPromptSlot(b, p[:-1])
    got = gpu.generateSampled([p[-1] for p in prompts], [len(p) - 1 for p in prompts], n_steps, cfgs,
                              [list(p) for p in prompts])
    for b in range(B):
        assert gpu.kvCache(b).size() == len(prompts[b]) - 1 + n_steps
    single = LlamaModel(LlamaConfig.fromShape(shape), t)
    want = host_loop(single, prompts, n_steps, cfgs)
    for b in range(B):
        assert got[b].tolist() == want[b], b


@pytest.mark.parametrize("ffn", [512, 480], ids=["batched-prompt", "prompt-in-steps"])
def test_scheduler_matches_serial_generation(ffn, cuda):
    """Six requests over four slots (two wait for a free slot), different
    prompt lengths, budgets, sampler settings and an EOS stop, against each
    request generated alone. With FFN 480 the model has no batched prompt
    path, so prompts run token by token inside the batched steps."""
    shape = dataclasses.replace(synth.TINY, ffn=ffn)
    t = synth.generate_numpy(shape, seed=62)
    gpu = LlamaModel(LlamaConfig.fromShape(shape), t, max_batch=4)
    reqs = []
    for i in range(6):
        prompt = synth.prompt_ids(shape, 70 + i, 3 + 4 * i).tolist()
        cfg = [SamplerConfig(0.7, 40, 0.95, 1.1, 21 + i), SamplerConfig(0.0, 1, 1.0, 1.0, 1),
               SamplerConfig(1.2, 8, 1.0, 1.2, 31 + i)][i % 3]
        reqs.append((prompt, 6 + 3 * i, cfg))
    single = LlamaModel(LlamaConfig.fromShape(shape), t)
    serial = [host_loop(single, [p], n, [c])[0] for p, n, c in reqs]
    eos = serial[4][3]  # request 4 stops at its 4th token, unemitted
    sched = BatchScheduler(gpu)
    ids = [sched.submit(p, n, c, eosTokenId=eos if i == 4 else -1) for i, (p, n, c) in enumerate(reqs)]
    steps = sched.runToCompletion(max_steps=500)
    assert steps < 500
    for i, rid in enumerate(ids):
        out, done = sched.result(rid)
        want = serial[i][: serial[i].index(eos)] if i == 4 else serial[i]
        assert done
        assert out.tolist() == want, i
    sched.close()


def test_scheduler_rejects_requests_beyond_context(cuda):
    gpu = sampler_model(1000)
    sched = BatchScheduler(gpu)
    ctx = synth.TINY.ctx
    with pytest.raises(_lib.IllegalArgumentException):
        sched.submit([1] * (ctx - 3), 4, SamplerConfig.greedy())
    rid = sched.submit([1] * (ctx - 4), 4, SamplerConfig.greedy())
    sched.runToCompletion(max_steps=20)
    out, done = sched.result(rid)
    assert done and out.size == 4
    sched.close()
