"""Tensor-parallel partition plan checked across 2 gloo ranks on CPU.

Each rank computes its Megatron shard of one decoder layer with the oracle's
arithmetic (wq/wk/wv by heads, wo by input rows, w1/w3 by output rows, w2 by
input columns, lm_head by vocabulary rows); the all-reduces and the logits
all-gather run over gloo. The result must equal the unsharded oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from auratensor_b200 import synth, tp
from oracle import ref


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer_tp(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shape = synth.TINY
        t = synth.generate_numpy(shape, seed=11)
        cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                              shape.rope_theta, shape.eps, shape.vocab)
        full = ref.LlamaModelRef(cfg, t)
        plan = tp.shard_plan(shape.n_heads, shape.n_kv_heads, shape.ffn, shape.vocab, world)
        rr = plan["ranges"][rank]
        hd = cfg.head_dim
        lw = full.layers[0]
        x = full.tok_embd[7].copy()
        ref.rmsnorm_inplace(x, lw["attn_norm.weight"], cfg.rms_norm_eps)
        q0, q1 = rr["q_cols"]
        k0, k1 = rr["kv_heads"]
        wq = lw["attn_q.weight"][:, q0 * hd:q1 * hd]
        wo = lw["attn_output.weight"][q0 * hd:q1 * hd, :]
        wv = lw["attn_v.weight"][:, k0 * hd:k1 * hd]
        # with one position the attention output of each head is its v (softmax of one score)
        qh = x @ wq
        vh = x @ wv
        g = (q1 - q0) // (k1 - k0)
        att = np.concatenate([vh[(h // g) * hd:(h // g + 1) * hd] for h in range(q1 - q0)])
        part = (att @ wo).astype(np.float32)
        y = torch.from_numpy(part.copy())
        dist.all_reduce(y)
        x2 = (x + y.numpy()).astype(np.float32)
        ref.rmsnorm_inplace(x2, lw["ffn_norm.weight"], cfg.rms_norm_eps)
        f0, f1 = rr["ffn"]
        gt = ref.sgemv(lw["ffn_gate.weight"][f0:f1], x2)
        up = ref.sgemv(lw["ffn_up.weight"][f0:f1], x2)
        ref.silu_inplace(gt)
        hpart = (gt * up).astype(np.float32)
        dpart = ref.sgemv(np.ascontiguousarray(lw["ffn_down.weight"][:, f0:f1]), hpart)
        y2 = torch.from_numpy(dpart.copy())
        dist.all_reduce(y2)
        out = (x2 + y2.numpy()).astype(np.float32)
        v0, v1 = rr["vocab"]
        lg = ref.sgemv(full.out_w[v0:v1], out)
        pad = np.zeros(plan["vocab_rows"], dtype=np.float32)
        pad[: v1 - v0] = lg
        gathered = [torch.zeros(plan["vocab_rows"]) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(pad))
        logits = torch.cat(gathered).numpy()[: shape.vocab]
        obj = [b"x" * 128 if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        q.put((rank, out, logits, qh, obj[0]))
    finally:
        dist.destroy_process_group()


def test_layer_tp_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_layer_tp, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # unsharded oracle of the same single-layer, single-position computation
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=11)
    cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                          shape.rope_theta, shape.eps, shape.vocab)
    full = ref.LlamaModelRef(cfg, t)
    lw = full.layers[0]
    x = full.tok_embd[7].copy()
    ref.rmsnorm_inplace(x, lw["attn_norm.weight"], cfg.rms_norm_eps)
    hd = cfg.head_dim
    v = x @ lw["attn_v.weight"]
    g = cfg.head_count // cfg.head_count_kv
    att = np.concatenate([v[(h // g) * hd:(h // g + 1) * hd] for h in range(cfg.head_count)])
    x2 = (x + att @ lw["attn_output.weight"]).astype(np.float32)
    ref.rmsnorm_inplace(x2, lw["ffn_norm.weight"], cfg.rms_norm_eps)
    gt = ref.sgemv(lw["ffn_gate.weight"], x2)
    up = ref.sgemv(lw["ffn_up.weight"], x2)
    ref.silu_inplace(gt)
    out = (x2 + ref.sgemv(lw["ffn_down.weight"], (gt * up).astype(np.float32))).astype(np.float32)
    logits = ref.sgemv(full.out_w, out)
    for rank, o, lg, _, uid in res:
        np.testing.assert_allclose(o, out, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(lg, logits, rtol=1e-4, atol=1e-4)
        assert uid == b"x" * 128


def test_shard_plan_rejects_bad_splits():
    with pytest.raises(ValueError):
        tp.shard_plan(32, 8, 14336, 128256, 3)
    p = tp.shard_plan(64, 8, 28672, 128256, 8)
    assert p["kv_heads"] == 1 and p["ffn"] == 3584 and p["vocab_rows"] == 16032
