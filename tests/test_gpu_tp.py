"""Tensor parallelism on 2 GPUs (Megatron shards; the per-layer all-reduces
and the logits gather are the library's own kernels over NVLink peer memory,
captured in the step graph) against the unsharded oracle.

Two child processes, one per GPU, build the same tiny model from the same
tensors with ``world=2``; rank 0 compares its logits with the oracle at every
teacher-forced step (1e-3 x logit range, the FP32 path tolerance). Skipped
when fewer than 2 GPUs are visible. NVLS is disabled so no rank ever binds
memory to an NVLink multicast object.
"""
import os
import socket

import numpy as np
import pytest
import torch

from auratensor_b200 import synth

pytestmark = pytest.mark.gpu
REL_TOL = 1e-3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, shape_name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist
    from auratensor_b200 import _lib, tp
    from auratensor_b200.inference import LlamaConfig, LlamaModel
    from oracle import ref

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ctx = None
    model = None
    try:
        shape = getattr(synth, shape_name)
        t = synth.generate_numpy(shape, seed=5)
        prompt = synth.prompt_ids(shape, 5, 8).tolist()
        ctx, r, w = tp.init_tp_context(rank)
        model = LlamaModel(LlamaConfig.fromShape(shape), t, ctx=ctx, world=w)
        orc = None
        if rank == 0:
            cfg = ref.LlamaConfig(shape.ctx, shape.dim, shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.ffn,
                                  shape.rope_theta, shape.eps, shape.vocab)
            orc = ref.LlamaModelRef(cfg, t)
        toks = list(prompt)
        worst = 0.0
        for pos in range(len(prompt) + 8):
            lg = model.forwardStep(toks[pos], pos).copy()
            nxt = [0]
            if rank == 0:
                lr = orc.forward_step(toks[pos], pos)
                rng_ = float(lr.max() - lr.min())
                worst = max(worst, float(np.max(np.abs(lg - lr))) / rng_)
                nxt = [int(np.argmax(lr))]
            obj = [nxt[0]]
            dist.broadcast_object_list(obj, src=0)
            if len(toks) < len(prompt) + 8 and pos >= len(prompt) - 1:
                toks.append(obj[0])
        q.put((rank, worst, None))
    except Exception as e:  # reported to the parent; every rank still tears down in order
        q.put((rank, None, repr(e)))
    finally:
        if model is not None:
            model.close()
        if ctx is not None:
            _lib.call("at_ctx_destroy", ctx)
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shape_name", ["TINY", "TINY_Q8"])
def test_tp2_matches_unsharded_oracle(shape_name):
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, shape_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, worst, err = q.get(timeout=300)
        res[rank] = (worst, err)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][1] is None and res[1][1] is None, res
    assert res[0][0] <= REL_TOL, res[0][0]


def _rank_stall(rank, world, port, q):
    """Rank 1 builds the model but never runs a step: rank 0's all-reduce wait
    must end at its bound with an error, not hang."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch.distributed as dist
    from auratensor_b200 import _lib, tp
    from auratensor_b200.inference import LlamaConfig, LlamaModel

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ctx = model = None
    try:
        shape = synth.TINY
        t = synth.generate_numpy(shape, seed=6)
        ctx, _, w = tp.init_tp_context(rank)
        model = LlamaModel(LlamaConfig.fromShape(shape), t, ctx=ctx, world=w)
        dist.barrier()
        outcome = "no step"
        if rank == 0:
            try:
                model.forwardStep(1, 0)
                outcome = "returned"
            except _lib.AtError as e:
                outcome = str(e)
        dist.barrier()
        q.put((rank, outcome))
    except Exception as e:
        q.put((rank, "exception: " + repr(e)))
    finally:
        if model is not None:
            model.close()
        if ctx is not None:
            _lib.call("at_ctx_destroy", ctx)
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_peer_that_never_arrives_fails_the_step():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_stall, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert "did not arrive" in res[0], res
