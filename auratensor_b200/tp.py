"""Tensor-parallel bootstrap: one process per GPU, torch.distributed for the
rendezvous, an NCCL communicator owned by libauratensor_cuda.so that
exchanges the peer-memory handles once at model finalize (the per-layer
all-reduces and the logits gather are the library's own kernels over NVLink
peer memory).

Rank 0 creates the 128-byte NCCL unique id through the C ABI and broadcasts
it with ``torch.distributed``; every rank then creates its ``at_ctx`` with
``at_ctx_create_tp``. Weight sharding (Megatron: wq/wk/wv and w1/w3 by output,
wo and w2 by input, lm_head by vocabulary rows) happens inside
``at_model_set_tensor`` from the full tensors every rank is given.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from ._lib import ModelConfig, ShardRegion, call


def shard_plan(n_heads: int, n_kv_heads: int, ffn: int, vocab: int, world: int) -> dict:
    """Per-rank shares the library cuts (mirrors at_model_create's checks)."""
    if n_kv_heads % world:
        raise ValueError("KV heads must divide evenly across tensor-parallel ranks")
    if ffn % (32 * world):
        raise ValueError("FFN width must split into 32-aligned shards")
    vl = (vocab + world - 1) // world
    return {
        "q_heads": n_heads // world,
        "kv_heads": n_kv_heads // world,
        "ffn": ffn // world,
        "vocab_rows": vl,
        "ranges": {
            r: {
                "q_cols": (r * (n_heads // world), (r + 1) * (n_heads // world)),
                "kv_heads": (r * (n_kv_heads // world), (r + 1) * (n_kv_heads // world)),
                "ffn": (r * (ffn // world), (r + 1) * (ffn // world)),
                "vocab": (r * vl, min(vocab, (r + 1) * vl)),
            }
            for r in range(world)
        },
    }


def shard_region(cfg: ModelConfig, world: int, rank: int, tensor_name: str) -> ShardRegion:
    """The part of a GGUF tensor rank ``rank`` keeps, as the library's upload
    cuts it (``at_tp_shard_region``: host-only, no GPU needed)."""
    out = ShardRegion()
    call("at_tp_shard_region", C.byref(cfg), world, rank, tensor_name.encode(), C.byref(out))
    return out


def unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    call("at_tp_unique_id", buf)
    return bytes(buf)


def init_tp_context(device: int | None = None, group=None):
    """Creates this rank's at_ctx over an NCCL communicator of the whole group.

    Requires torch.distributed to be initialised. Returns (ctx, rank, world).
    """
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if device is None:
        device = torch.cuda.current_device()
    obj = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = (C.c_uint8 * 128).from_buffer_copy(obj[0])
    ctx = C.c_void_p()
    call("at_ctx_create_tp", device, rank, world, uid, C.byref(ctx))
    return ctx.value, rank, world
