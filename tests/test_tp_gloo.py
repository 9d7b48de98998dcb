"""Tensor-parallel partition checked across 2 and 4 gloo ranks on CPU.

Every rank asks the library (``at_tp_shard_region``, the same function its
upload uses to cut a rank's shard) which part of each weight tensor it keeps
and where that part lands in its device matrices, cuts its shard of one
decoder layer that way from the full tensors, and runs the layer with the
oracle's arithmetic on those local matrices (fused [q|k|v], wo by head rows,
w1/w3 by output rows, w2 by input columns, lm_head by vocabulary rows). The
all-reduces and the logits all-gather run over gloo. The result must equal
the unsharded oracle, for the reference's [in][out] attention and for
llama.cpp's [out][in].
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from auratensor_b200 import _lib, synth, tp
from oracle import ref

# 8 query / 4 KV heads of 64, FFN 1024 (32-aligned shards at 4 ranks) and a
# vocabulary of 1001 rows, so the last rank's lm_head share is short
SHAPE = synth.ModelShape("tp-layer", 1, 512, 1024, 8, 4, 1001, 10000.0, 16, synth.Q4_0)
TOKEN = 7


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    t = synth.generate_numpy(SHAPE, seed=11)
    cfg = ref.LlamaConfig(SHAPE.ctx, SHAPE.dim, SHAPE.n_layers, SHAPE.n_heads, SHAPE.n_kv_heads, SHAPE.ffn,
                          SHAPE.rope_theta, SHAPE.eps, SHAPE.vocab)
    return cfg, ref.LlamaModelRef(cfg, t)


def _c_config(layout):
    return _lib.ModelConfig(SHAPE.ctx, SHAPE.dim, SHAPE.n_layers, SHAPE.n_heads, SHAPE.n_kv_heads, SHAPE.ffn,
                            SHAPE.vocab, SHAPE.rope_theta, SHAPE.eps, 1, layout, 0, 0)


def _logical(full, lw, name, attn_out_in):
    """The tensor as its bytes are laid out ([rows][cols]), dequantized."""
    if name == "output.weight":
        return full.out_w
    w = lw[name.split(".", 2)[-1] if name.startswith("blk.") else name]
    if attn_out_in and "attn_" in name:
        return np.ascontiguousarray(w.T)
    return w


def _cut(cfg_c, world, rank, name, full_t, locals_):
    """Copies this rank's part of full_t into its device matrix, as the upload does."""
    rg = tp.shard_region(cfg_c, world, rank, name)
    assert full_t.shape == (rg.rows, rg.cols), name
    key = rg.target
    if key not in locals_:
        locals_[key] = (rg.orient, np.zeros((rg.local_rows, rg.local_cols), dtype=np.float32))
    orient, dst = locals_[key]
    assert orient == rg.orient and dst.shape == (rg.local_rows, rg.local_cols), name
    dst[rg.dst_row0:rg.dst_row0 + rg.n_rows, rg.dst_col0:rg.dst_col0 + rg.n_cols] = \
        full_t[rg.src_row0:rg.src_row0 + rg.n_rows, rg.src_col0:rg.src_col0 + rg.n_cols]
    return rg


def _apply(mat, x):
    orient, w = mat
    return ref.sgemv(w, x) if orient == _lib.ORIENT_N else (x.astype(np.float64) @ w).astype(np.float32)


def _layer_tp(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, full = _model()
        lw = full.layers[0]
        hd = cfg.head_dim
        results = {}
        for layout in (_lib.LAYOUT_REFERENCE, _lib.LAYOUT_ATTN_OUT_IN):
            attn_out_in = layout == _lib.LAYOUT_ATTN_OUT_IN
            cfg_c = _c_config(layout)
            mats = {}
            for name in ("blk.0.attn_q.weight", "blk.0.attn_k.weight", "blk.0.attn_v.weight",
                         "blk.0.attn_output.weight", "blk.0.ffn_gate.weight", "blk.0.ffn_up.weight",
                         "blk.0.ffn_down.weight", "output.weight"):
                _cut(cfg_c, world, rank, name, _logical(full, lw, name, attn_out_in), mats)
            for name in ("blk.0.attn_norm.weight", "token_embd.weight", "output_norm.weight"):
                assert tp.shard_region(cfg_c, world, rank, name).n_rows == \
                    tp.shard_region(cfg_c, world, rank, name).rows  # whole on every rank
            assert tp.shard_region(cfg_c, world, rank, "rope_freqs.weight").target == _lib.SHARD_NONE
            x = full.tok_embd[TOKEN].copy()
            ref.rmsnorm_inplace(x, lw["attn_norm.weight"], cfg.rms_norm_eps)
            qkv = _apply(mats[_lib.SHARD_QKV], x)
            Hl, Hkvl = cfg.head_count // world, cfg.head_count_kv // world
            v = qkv[(Hl + Hkvl) * hd:]
            g = Hl // Hkvl
            # one position: each head's attention output is its KV head's v
            att = np.concatenate([v[(h // g) * hd:(h // g + 1) * hd] for h in range(Hl)])
            y = torch.from_numpy(_apply(mats[_lib.SHARD_WO], att).copy())
            dist.all_reduce(y)
            x2 = (x + y.numpy()).astype(np.float32)
            ref.rmsnorm_inplace(x2, lw["ffn_norm.weight"], cfg.rms_norm_eps)
            gt = _apply(mats[_lib.SHARD_W1], x2)
            up = _apply(mats[_lib.SHARD_W3], x2)
            ref.silu_inplace(gt)
            y2 = torch.from_numpy(_apply(mats[_lib.SHARD_W2], (gt * up).astype(np.float32)).copy())
            dist.all_reduce(y2)
            out = (x2 + y2.numpy()).astype(np.float32)
            lg = torch.from_numpy(_apply(mats[_lib.SHARD_OUTPUT], out).copy())  # Vl rows, zero past the vocabulary
            gathered = [torch.zeros_like(lg) for _ in range(world)]
            dist.all_gather(gathered, lg)
            results[layout] = (out, torch.cat(gathered).numpy()[: cfg.vocab_size])
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def _unsharded():
    cfg, full = _model()
    lw = full.layers[0]
    x = full.tok_embd[TOKEN].copy()
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
    return out, ref.sgemv(full.out_w, out)


@pytest.mark.parametrize("world", [2, 4])
def test_layer_tp_matches_unsharded(world):
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
    out, logits = _unsharded()
    for rank, results in res:
        assert set(results) == {_lib.LAYOUT_REFERENCE, _lib.LAYOUT_ATTN_OUT_IN}
        for o, lg in results.values():
            np.testing.assert_allclose(o, out, rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(lg, logits, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_library_shards_agree_with_python_plan(world):
    # the 70B shape: 64/8 heads, FFN 28672, vocabulary 128256
    cfg_c = _lib.ModelConfig(8192, 8192, 80, 64, 8, 28672, 128256, 500000.0, 1e-5, 1, 0, 0, 0)
    plan = tp.shard_plan(64, 8, 28672, 128256, world)
    hd = 128
    for r in range(world):
        rr = plan["ranges"][r]
        q = tp.shard_region(cfg_c, world, r, "blk.5.attn_q.weight")
        assert (q.src_col0, q.n_cols) == (rr["q_cols"][0] * hd, (rr["q_cols"][1] - rr["q_cols"][0]) * hd)
        k = tp.shard_region(cfg_c, world, r, "blk.5.attn_k.weight")
        assert (k.src_col0, k.n_cols) == (rr["kv_heads"][0] * hd, (rr["kv_heads"][1] - rr["kv_heads"][0]) * hd)
        assert k.dst_col0 == q.n_cols and q.local_cols == q.n_cols + 2 * k.n_cols
        wo = tp.shard_region(cfg_c, world, r, "blk.5.attn_output.weight")
        assert (wo.src_row0, wo.n_rows, wo.n_cols) == (q.src_col0, q.n_cols, 8192)
        up = tp.shard_region(cfg_c, world, r, "blk.5.ffn_up.weight")
        assert (up.src_row0, up.src_row0 + up.n_rows) == rr["ffn"]
        down = tp.shard_region(cfg_c, world, r, "blk.5.ffn_down.weight")
        assert (down.src_col0, down.src_col0 + down.n_cols) == rr["ffn"] and down.n_rows == 8192
        out = tp.shard_region(cfg_c, world, r, "output.weight")
        assert (out.src_row0, out.src_row0 + out.n_rows) == rr["vocab"] and out.local_rows == plan["vocab_rows"]


def test_shard_plan_rejects_bad_splits():
    with pytest.raises(ValueError):
        tp.shard_plan(32, 8, 14336, 128256, 3)
    p = tp.shard_plan(64, 8, 28672, 128256, 8)
    assert p["kv_heads"] == 1 and p["ffn"] == 3584 and p["vocab_rows"] == 16032
    cfg_c = _lib.ModelConfig(2048, 4096, 32, 32, 8, 14336, 128256, 500000.0, 1e-5, 1, 0, 0, 0)
    with pytest.raises(_lib.IllegalArgumentException, match="KV heads"):
        tp.shard_region(cfg_c, 3, 0, "blk.0.attn_q.weight")
    with pytest.raises(_lib.IllegalArgumentException, match="rank"):
        tp.shard_region(cfg_c, 2, 2, "blk.0.attn_q.weight")
