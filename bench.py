"""Benchmark: Llama-3-8B-shaped Q4_0 batch-1 greedy decode (tokens/s) on B200.

Workload: random-init Llama-3-8B shape (32 layers, dim 4096, FFN 14336, 32/8
heads, head_dim 128, vocab 128256, RoPE theta 500000, context 2048), weights
N(0, 0.02) quantized to Q4_0 on the device, a seeded 512-token prompt run
through forwardPrompt (timed separately: the "prompt" object, median of 3
runs after a warm-up), then timed decode steps from position 512.
One step = one decode token. Weights (4.6 GB) exceed the 126 MB L2, so no
flush is needed between steps.

  value  device-resident greedy loop (at_model_generate), CUDA events on the
         engine's stream, max over ranks.
  e2e    the reference-facing call: at_model_forward_step with the token in
         and the full logits out in host memory each step, then the greedy
         Sampler on the host (the reference's decode loop).

N > 1: one process per GPU (torchrun), Megatron tensor parallelism; the
per-layer all-reduces and the logits gather are the library's own kernels over
NVLink peer memory (NCCL only exchanges the memory handles at load); scaling
"strong".

--config selects the other workloads (their own metric names):
  llama-3-70b              80 layers, dim 8192, Q4_0 (39.5 GB), 1024-token
                           prompt, greedy decode at context 8192.
  mistral-7b-q8_0-batch8   Mistral-7B shape, Q8_0, 8 requests with 128-token
                           seeded prompts, temperature 0.7 / top-k 40 / top-p
                           0.95 with fixed seeds, batched decode at context
                           4096; one step = one batched step (8 tokens).
                           value: at_model_generate_sampled (step graph +
                           device sampler + token feedback on the device);
                           e2e: the request scheduler (at_sched_step: tokens
                           and positions in, sampled ids out, every step).

--impl reference: the reference's CPU algorithm (load-time dequant to FP32,
FP32 sgemv; the C restatement under oracle/) on all host cores, each step a
sampled decode token (2 of the layers plus the lm_head, extrapolated); the
reference serves one request at a time, so its batch-8 rate is its
single-sequence rate (plus the host Sampler for the sampled workload).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

UNIT = "tok/s"
SAMPLE_LAYERS = 2
# workload name -> (shape name in synth, metric, prompt tokens, batch, sampler (T, topK, topP, penalty) or None)
CONFIGS = {
    "llama-3.2-1b": ("LLAMA32_1B", "Llama-3.2-1B Q4_0 decode tok/s", 8, 1, None),
    "llama-3-8b": ("LLAMA3_8B", "Llama-3-8B Q4_0 decode tok/s", 512, 1, None),
    "llama-3-70b": ("LLAMA3_70B", "Llama-3-70B Q4_0 decode tok/s", 1024, 1, None),
    "mistral-7b-q8_0-batch8": ("MISTRAL_7B", "Mistral-7B Q8_0 batch-8 sampled decode tok/s", 128, 8,
                               (0.7, 40, 0.95, 1.0)),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--profile-steps", type=int, default=8)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    p.add_argument("--config", default="llama-3-8b", choices=sorted(CONFIGS))
    p.add_argument("--kv-type", default="f32", choices=["f32", "q8_0"],
                   help="KV cache storage (q8_0: the quantized cache, a stated 2e-2 logit tolerance)")
    # smaller cases for profiler captures only (the bench line uses the defaults)
    p.add_argument("--prompt", type=int, default=None)
    p.add_argument("--layers", type=int, default=None)
    a = p.parse_args()
    shape_name, a.metric, prompt, a.batch, a.sampler = CONFIGS[a.config]
    a.kv = 8 if a.kv_type == "q8_0" else 0
    if a.kv:
        a.metric = a.metric.replace(" tok/s", " (Q8_0 KV) tok/s")
    a.shape_name = shape_name
    if a.prompt is None:
        a.prompt = prompt
    return a


def config_shape(args):
    import dataclasses
    from auratensor_b200 import synth
    shape = getattr(synth, args.shape_name)
    if args.layers is not None:
        shape = dataclasses.replace(shape, n_layers=args.layers)
    return shape


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
CLOCK_Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# algorithmic bytes per launch (weights + input vector + output vector)
# ---------------------------------------------------------------------------
def q_bytes(rows, cols, bpb=18):
    return rows * (cols // 32) * bpb


def class_bytes(shape, world, pos, batch=1, kv_type=0):
    """Algorithmic bytes of one step per kernel class: the quantized weights
    once, the activations in and out of every row, and each row's KV cache
    up to its position (pos: one position or one per row)."""
    d, hd = shape.dim, shape.head_dim
    hl, hkvl, fl = shape.n_heads // world, shape.n_kv_heads // world, shape.ffn // world
    vl = -(-shape.vocab // world)
    qkv_cols = (hl + 2 * hkvl) * hd
    bpb = 34 if shape.wtype == 8 else 18
    ps = list(pos) if isinstance(pos, (list, tuple)) else [pos] * batch
    kv_elem = 4 if kv_type == 0 else 1 + 2 / 32  # bytes per cached element (Q8_0: quant + shared fp16 scale)
    return {
        "qkv": q_bytes(d, qkv_cols, bpb) + batch * (d * 4 + qkv_cols * 4),
        "wo": q_bytes(hl * hd, d, bpb) + batch * (hl * hd * 4 + d * 4),
        "ffn_up": 2 * q_bytes(fl, d, bpb) + batch * (d * 4 + fl * 4),
        "ffn_down": q_bytes(d, fl, bpb) + batch * (fl * 4 + d * 4),
        "lm_head": q_bytes(vl, d, bpb) + batch * (d * 4 + vl * 4),
        "attn": sum(2 * hkvl * (p + 1) * hd * kv_elem + 2 * hl * hd * 4 for p in ps),
    }


def step_bytes_of(shape, world, positions_per_step, batch, kv_type=0):
    """Mean bytes one GPU must move per step over the timed steps."""
    tot = 0.0
    for pos in positions_per_step:
        cb = class_bytes(shape, world, pos, batch, kv_type)
        tot += shape.n_layers * (cb["qkv"] + cb["attn"] + cb["wo"] + cb["ffn_up"] + cb["ffn_down"])
        tot += cb["lm_head"] + batch * q_bytes(1, shape.dim, 34 if shape.wtype == 8 else 18)
    return tot / len(positions_per_step)


def prompt_flops(shape, n):
    """FLOPs of the batched prompt path for n tokens: every layer's QKV and
    attention (2 * 2 * H * hd * (p + 1) per token p), every layer but the
    last's wo and feed-forward (only the KV cache carries over to decode)."""
    d, hd, H, Hkv, F, L = shape.dim, shape.head_dim, shape.n_heads, shape.n_kv_heads, shape.ffn, shape.n_layers
    qcols = (H + 2 * Hkv) * hd
    linear = 2.0 * n * (L * d * qcols + (L - 1) * (H * hd * d + 3 * d * F))
    attn = 4.0 * H * hd * L * n * (n + 1) / 2
    return linear + attn


def time_prompt(run, stream, reduce, reps=3):
    """Median device (CUDA events on the engine's stream, reduced over ranks)
    and wall time of `reps` prompt runs after one untimed run (the first
    allocates the prompt buffers). A rerun rewrites the same KV positions."""
    import torch

    run()
    torch.cuda.synchronize()
    dev, wall = [], []
    for _ in range(reps):
        t0 = time.time()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        run()
        p1.record(stream)
        p1.synchronize()
        wall.append(time.time() - t0)
        dev.append(reduce(p0.elapsed_time(p1)) / 1000.0)
    return sorted(dev)[len(dev) // 2], sorted(wall)[len(wall) // 2]


def prompt_line(shape, world, n, dev_s, wall_s, requests=1):
    """The prompt's device time (CUDA events on the engine's stream) and, on
    one GPU (the tensor-core path), its FLOP rate against the bf16 peak."""
    out = {"tokens": n * requests, "seconds": round(dev_s, 4), "wall_seconds": round(wall_s, 4),
           "tok_s": round(n * requests / dev_s, 1) if dev_s > 0 else None}
    if world == 1 and dev_s > 0:
        peak = 1625.1
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peak = float(json.load(f)["bf16_tflops"])
        except (OSError, KeyError, ValueError):
            pass
        tf = prompt_flops(shape, n) * requests / dev_s / 1e12
        out.update({"path": "tcgen05 bf16 GEMMs and attention, 512-token chunks", "tflops": round(tf, 1),
                    "peak_tflops": peak, "frac": round(tf / peak, 4)})
    else:
        out["path"] = "decode steps (tensor parallel)"
    return out


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ---------------------------------------------------------------------------
# CPU baseline: the reference algorithm (C restatement) on a sampled token
# ---------------------------------------------------------------------------
def cpu_decode_sample(shape, host_tensors, threads, steps, start_pos):
    """Time `steps` decode tokens of the reference algorithm with SAMPLE_LAYERS
    layers, extrapolated to all layers. Returns (tok/s list per step, detail)."""
    from oracle.cref import RefDecoder
    dec = RefDecoder(shape, n_layers=SAMPLE_LAYERS, threads=threads)
    for name, (tt, data, numel) in host_tensors.items():
        dec.set_tensor(name, tt, data, numel)
    rates = []
    tok = 1
    for i in range(steps):
        dec.forward_step(tok, start_pos + i)
        te, tl, th = dec.times()
        t_tok = te + tl * (shape.n_layers / SAMPLE_LAYERS) + th
        rates.append(1.0 / t_tok)
    dec.close()
    return rates


def sample_host_tensors_cpu(shape, seed):
    """Synthetic Q4_0 tensors of the sampled layers, generated on the CPU."""
    import torch
    from auratensor_b200 import synth
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, dims, t in shape.tensor_dims():
        if name.startswith("blk.") and int(name.split(".")[1]) >= SAMPLE_LAYERS:
            continue
        n = int(np.prod(dims))
        if t == 0:
            data = np.ones(n, dtype=np.float32).view(np.uint8)
        else:
            parts = []
            step = 1 << 25
            for s0 in range(0, n, step):
                c = min(step, n - s0)
                x = torch.randn(c, generator=g, dtype=torch.float32) * 0.02
                parts.append(synth.quantize_torch(x, t).numpy())
            data = np.concatenate(parts)
        out[name] = (t, data, n)
    return out


def host_sampler_seconds(vocab, cfg, reps=20):
    """Seconds per call of the host Sampler (native restatement) on one
    vocab-sized logits row with the workload's settings."""
    from auratensor_b200.inference import Sampler, SamplerConfig
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(vocab) * 3).astype(np.float32)
    t, k, p, rp = cfg
    c = SamplerConfig(t, k, p, rp, 1234)
    t0 = time.perf_counter()
    for _ in range(reps):
        Sampler.sample(x.copy(), None, c)
    return (time.perf_counter() - t0) / reps


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shape = config_shape(args)
    threads = os.cpu_count() or 1
    t0 = time.time()
    tensors = sample_host_tensors_cpu(shape, args.seed)
    gen_s = time.time() - t0
    rates = cpu_decode_sample(shape, tensors, threads, args.warmup + args.steps, args.prompt)
    timed = rates[args.warmup:]
    sec_per_tok = sum(1.0 / r for r in timed) / len(timed)
    sampler_s = 0.0
    if args.sampler is not None:
        sampler_s = host_sampler_seconds(shape.vocab, args.sampler)
    value = 1.0 / (sec_per_tok + sampler_s)
    sample = (f"{SAMPLE_LAYERS} of {shape.n_layers} layers + lm_head per step, decode positions "
              f"{args.prompt}..{args.prompt + args.warmup + args.steps - 1}, extrapolated to {shape.n_layers} layers")
    if args.sampler is not None:
        sample += (f"; one request at a time as the reference's server (its batch-{args.batch} rate is its "
                   f"single-sequence rate), plus the host Sampler ({sampler_s * 1e3:.3f} ms per token)")
    line = {
        "metric": args.metric, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000.0 / value, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": workload_name(args, shape), "batch": args.batch, "prompt_tokens": args.prompt,
                   "context": shape.ctx,
                   "weights": f"{'Q8_0' if shape.wtype == 8 else 'Q4_0'} dequantized to FP32 at load "
                              "(reference algorithm)"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample, "setup_s": round(gen_s, 1)},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_name(args, shape):
    q = "q8_0" if shape.wtype == 8 else "q4_0"
    base = args.config if q in args.config else f"{args.config}-{q}"
    return base + ("-sampled-decode" if args.sampler is not None else "-decode")


# ---------------------------------------------------------------------------
# our engine
# ---------------------------------------------------------------------------
def build_model(shape, seed, ctx, world, keep_host: bool, max_batch: int = 1, kv_type: int = 0):
    import torch
    from auratensor_b200 import synth
    from auratensor_b200.inference import LlamaConfig, LlamaModel
    model = LlamaModel(LlamaConfig.fromShape(shape), None, max_batch=max_batch, ctx=ctx, world=world,
                       kv_type=kv_type)
    g = torch.Generator(device="cuda").manual_seed(seed)
    host = {}
    for name, dims, t in shape.tensor_dims():
        data = synth.generate_torch_tensor(dims, t, g, "cuda")
        model.setTensor(name, t, data)
        if keep_host and (not name.startswith("blk.") or int(name.split(".")[1]) < SAMPLE_LAYERS):
            host[name] = (t, data.cpu().numpy(), int(np.prod(dims)))
        del data
    model.finalize()
    torch.cuda.synchronize()
    return model, host


def parity_check(full_shape, seed, ctx, world, rank, kv_type=0):
    """The bench's decode path against the oracle, in the same run and at the
    same tensor-parallel degree: a 2-layer model of the bench's dimensions
    (the same kernels and shard sizes) on every rank, and the C restatement
    of the reference on rank 0 with the same weights. The oracle runs 8
    seeded prompt tokens then 16 greedy steps; rank 0 broadcasts that token
    sequence, every rank steps the device model through it, and rank 0
    compares the logits of every step: max |delta| / (max - min of the
    oracle's logits) against the 1e-3 rule, and the greedy tokens (equal, or
    the oracle's top-2 gap below the rule)."""
    import dataclasses
    import torch
    import torch.distributed as dist
    from auratensor_b200 import synth
    from auratensor_b200.inference import LlamaConfig, LlamaModel
    shape = dataclasses.replace(full_shape, n_layers=2, ctx=64)
    n_prompt, n_greedy, tol = 8, 16, 1e-3
    g = torch.Generator(device="cuda").manual_seed(seed + 1000)
    model = LlamaModel(LlamaConfig.fromShape(shape), None, max_batch=1, ctx=ctx, world=world, kv_type=kv_type)
    orc = None
    if rank == 0:
        from oracle.cref import RefDecoder
        orc = RefDecoder(shape, threads=os.cpu_count() or 1, kv_type=kv_type)
    for name, dims, t in shape.tensor_dims():
        data = synth.generate_torch_tensor(dims, t, g, "cuda")
        model.setTensor(name, t, data)
        if orc is not None:
            orc.set_tensor(name, t, data.cpu().numpy(), int(np.prod(dims)))
        del data
    model.finalize()
    n = n_prompt + n_greedy
    seq = torch.zeros(n, dtype=torch.int64, device="cuda")
    ref_logits = []
    if rank == 0:
        toks = [int(v) for v in synth.prompt_ids(shape, seed, n_prompt)]
        for pos in range(n):
            lr = orc.forward_step(toks[pos], pos)
            ref_logits.append(lr)
            if pos + 1 < n and pos + 1 >= n_prompt:
                toks.append(int(np.argmax(lr)))
        seq.copy_(torch.tensor(toks, dtype=torch.int64))
        orc.close()
    if world > 1:
        dist.broadcast(seq, 0)
    toks = [int(v) for v in seq.cpu().tolist()]
    worst, equal, rule_ok = 0.0, 0, True
    for pos in range(n):
        lg = model.forwardStep(toks[pos], pos)
        if rank == 0:
            lr = ref_logits[pos]
            rng_ = float(lr.max() - lr.min())
            worst = max(worst, float(np.max(np.abs(lg - lr))) / rng_)
            if pos >= n_prompt - 1:
                if int(np.argmax(lg)) == int(np.argmax(lr)):
                    equal += 1
                else:
                    srt = np.sort(lr)
                    rule_ok = rule_ok and float(srt[-1] - srt[-2]) < tol * rng_
    model.close()
    return {"checked": True, "model": f"{shape.name} dims, 2 layers, tp{world}", "steps": n,
            "max_rel_err": float(f"{worst:.3g}"), "tol": tol, "greedy_steps": n_greedy + 1,
            "tokens_equal": equal, "passed": bool(worst <= tol and rule_ok)}


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from auratensor_b200 import _lib, build as libbuild, synth, tp
    from auratensor_b200.inference import Sampler, SamplerConfig

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    libbuild.build()
    torch.cuda.set_device(local)
    import ctypes as C
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        ctx, _, _ = tp.init_tp_context(local)
    else:
        p = C.c_void_p()
        _lib.call("at_ctx_create", local, C.byref(p))
        ctx = p.value
    shape = config_shape(args)
    if args.batch > 1:
        run_batched(args, shape, ctx, world, rank, local)
        return
    PROMPT = args.prompt
    keep_host = (rank == 0 and world == 1 and not args.no_cpu_baseline and args.layers is None)
    t0 = time.time()
    model, host = build_model(shape, args.seed, ctx, world, keep_host, kv_type=args.kv)
    load_s = time.time() - t0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    prompt = synth.prompt_ids(shape, args.seed, PROMPT).tolist()
    stream = torch.cuda.ExternalStream(model.stream())
    prefill_dev_s, prefill_s = time_prompt(lambda: model.forwardPrompt(prompt), stream, max_over_ranks)
    ctx_len = shape.ctx

    def positions(start, n):
        """Segments of consecutive positions in [start, ctx); wraps back to PROMPT."""
        segs, p, left = [], start, n
        while left:
            if p >= ctx_len:
                p = PROMPT
            k = min(left, ctx_len - p)
            segs.append((p, k))
            p += k
            left -= k
        return segs, p

    tok = int(prompt[-1])
    segs, pos = positions(args.prompt, args.warmup)
    for p0, k in segs:
        model.generate(tok, p0, k)
    gpus = list(range(torch.cuda.device_count()))[: max(1, world)] if world > 1 else [local]

    with ClockSampler(gpus) as clk:
        # value: device-resident greedy loop
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        segs, pos = positions(pos, args.steps)
        timed_pos = [p0 + i for p0, k in segs for i in range(k)]
        e0.record(stream)
        for p0, k in segs:
            model.generate(tok, p0, k, wait=False)
        e1.record(stream)
        e1.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1))
        # e2e: forwardStep with host logits + host greedy sampler, every step
        barrier()
        greedy = SamplerConfig.greedy()
        segs2, pos2 = positions(pos, args.steps)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        t = tok
        for p0, k in segs2:
            for i in range(k):
                logits = model.forwardStep(t, p0 + i)
                t = Sampler.sample(logits, None, greedy)
        f1.record(stream)
        f1.synchronize()
        ms_e2e = max_over_ranks(f0.elapsed_time(f1))
    clocks = clk.summary()
    pos = pos2

    # roofline: eager per-class kernel times over a few steps
    tot = {}
    for i in range(args.profile_steps):
        p = pos if pos < ctx_len else PROMPT
        r = model.profileStep(tok, p)
        pos = p + 1
        for k, (msk, n) in r.items():
            a = tot.setdefault(k, [0.0, 0])
            a[0] += msk
            a[1] += n
    value = args.steps / (ms / 1000.0)
    e2e = args.steps / (ms_e2e / 1000.0)
    parity = None
    if not args.no_parity:
        parity = parity_check(shape, args.seed, ctx, world, rank, args.kv)
    if rank != 0:
        finish(model, ctx, world)
        return
    bytes_per = class_bytes(shape, world, pos, 1, args.kv)
    # bytes one GPU must move per decode step (weights of its shards, its KV
    # heads at the timed positions, activations), over the measured step time
    step_bytes = step_bytes_of(shape, world, timed_pos, 1, args.kv)
    gemv = {k: v for k, v in tot.items() if k in bytes_per}
    dom = max(gemv, key=lambda k: gemv[k][0])
    avg_ms = gemv[dom][0] / max(1, gemv[dom][1])
    peak, peak_kind = load_peaks()
    achieved = bytes_per[dom] / (avg_ms / 1000.0) / 1e9
    # the committed capture is of the default workload (Llama-3-8B, fp32 KV, one GPU)
    traffic = committed_traffic().get(dom) if (args.config == "llama-3-8b" and not args.kv and world == 1) else None
    step_ms_eager = sum(v[0] for v in tot.values()) / args.profile_steps
    # embed; per layer QKV, attention (split + merge in one launch), wo, gate/up, down (+ two
    # all-reduces under TP); lm_head, argmax (2), greedy advance (+ logits gather under TP)
    launches_per_step = 1 + (5 + (2 if world > 1 else 0)) * shape.n_layers + 4 + (1 if world > 1 else 0)

    cpu = None
    if keep_host:
        threads = os.cpu_count() or 1
        rates = cpu_decode_sample(shape, host, threads, 4, PROMPT + 64)
        rates1 = cpu_decode_sample(shape, host, 1, 2, PROMPT + 64)
        cpu = {"value": round(len(rates) / sum(1 / r for r in rates), 4), "unit": UNIT, "cores": threads,
               "kind": "port",
               "sample": f"{SAMPLE_LAYERS} of {shape.n_layers} layers + lm_head, 4 decode tokens at positions "
                         f"{PROMPT + 64}.., extrapolated to {shape.n_layers} layers; same Q4_0 weights",
               "single_thread_value": round(len(rates1) / sum(1 / r for r in rates1), 4)}

    wbytes = sum(int(np.prod(dims)) // 32 * 18 for _, dims, t in shape.tensor_dims() if t != 0)
    line = {
        "metric": args.metric, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args, shape), "batch": 1, "prompt_tokens": PROMPT, "context": ctx_len,
                   "weights": f"Q4_0 ({wbytes / 1e9:.1f} GB, > L2; no flush needed)", "parallelism": f"tp{world}",
                   "kv_cache": args.kv_type, "seed": args.seed},
        "e2e": {"value": round(e2e, 3), "unit": UNIT, "h2d_bytes_per_step": 12,
                "d2h_bytes_per_step": shape.vocab * 4},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic, "bytes_per_launch": bytes_per[dom],
                     "avg_launch_us": round(avg_ms * 1000.0, 2),
                     "step_bytes": int(step_bytes),
                     "step_frac": round(step_bytes / (ms / args.steps / 1000.0) / 1e9 / peak, 4)},
        "parity": parity,
        "kernel_ms_per_step": {k: round(v[0] / args.profile_steps, 4) for k, v in tot.items() if v[1]},
        "eager_step_ms": round(step_ms_eager, 4),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "setup": {"load_s": round(load_s, 1), "prefill_s": round(prefill_s, 2)},
        # the prompt outside the decode timing (forwardPrompt: tcgen05 GEMMs over 512-token chunks on one
        # GPU), median of 3 runs after one warm-up, CUDA events
        "prompt": prompt_line(shape, world, args.prompt, prefill_dev_s, prefill_s),
    }
    print(json.dumps(line), flush=True)
    finish(model, ctx, world)


def batched_parity(full_shape, seed, ctx, batch, sampler, kv_type=0):
    """The batched sampled path against the oracle in the same run: a 2-layer
    model of the workload's dimensions with `batch` slots. Every row decodes
    its own 6-token seeded prompt and then 10 sampled tokens, all rows in one
    batched step each time (the device sampler picks the tokens, each row
    with its own seed and its prompt-plus-output penalty history). Each row
    is then replayed through the C restatement of the reference, teacher
    forced on the device's tokens: the logits must be within 1e-3 of the
    oracle's range at every step, the device sampler must pick what the host
    Sampler picks from the device's logits (exact), and the count of steps
    where the host Sampler on the oracle's logits picks the same id is
    reported."""
    import dataclasses
    import torch
    from auratensor_b200 import synth
    from auratensor_b200.inference import LlamaConfig, LlamaModel, Sampler, SamplerConfig
    from oracle.cref import RefDecoder
    shape = dataclasses.replace(full_shape, n_layers=2, ctx=64)
    n_prompt, n_gen, tol = 6, 10, 1e-3
    g = torch.Generator(device="cuda").manual_seed(seed + 2000)
    model = LlamaModel(LlamaConfig.fromShape(shape), None, max_batch=batch, ctx=ctx, kv_type=kv_type)
    orc = RefDecoder(shape, threads=os.cpu_count() or 1, kv_type=kv_type)
    for name, dims, t in shape.tensor_dims():
        data = synth.generate_torch_tensor(dims, t, g, "cuda")
        model.setTensor(name, t, data)
        orc.set_tensor(name, t, data.cpu().numpy(), int(np.prod(dims)))
        del data
    model.finalize()
    T, K, P, R = sampler
    cfgs = [SamplerConfig(T, K, P, R, 1000 + b) for b in range(batch)]
    prompts = [[int(v) for v in synth.prompt_ids(shape, seed + b, n_prompt)] for b in range(batch)]
    seqs = [list(p) for p in prompts]
    dev_logits = [[] for _ in range(batch)]
    sampler_equal = True
    for pos in range(n_prompt + n_gen - 1):
        toks = [seqs[b][pos] for b in range(batch)]
        lg = model.forwardBatch(toks, [pos] * batch).copy()
        if pos >= n_prompt - 1:
            got = model.sample(cfgs, seqs)
            for b in range(batch):
                dev_logits[b].append(lg[b].copy())
                want = Sampler.sample(lg[b].copy(), seqs[b], cfgs[b])
                sampler_equal = sampler_equal and int(got[b]) == want
                seqs[b].append(int(got[b]))
        else:
            for b in range(batch):
                dev_logits[b].append(lg[b].copy())
    worst, agree, total = 0.0, 0, 0
    for b in range(batch):
        for pos in range(n_prompt + n_gen - 1):
            lr = orc.forward_step(seqs[b][pos], pos)
            lg = dev_logits[b][pos]
            worst = max(worst, float(np.max(np.abs(lg - lr))) / float(lr.max() - lr.min()))
            if pos >= n_prompt - 1:
                total += 1
                agree += int(Sampler.sample(lr.copy(), seqs[b][:pos + 1], cfgs[b]) == seqs[b][pos + 1])
    orc.close()
    model.close()
    return {"checked": True, "model": f"{shape.name} dims, 2 layers, batch {batch}", "steps": n_prompt + n_gen - 1,
            "max_rel_err": float(f"{worst:.3g}"), "tol": tol, "sampled_steps": total,
            "device_sampler_equals_host": sampler_equal, "oracle_logits_same_token": agree,
            "passed": bool(worst <= tol and sampler_equal)}


def run_batched(args, shape, ctx, world, rank, local):
    """Batched sampled decode: value from at_model_generate_sampled over the
    batch (device loop), e2e from the request scheduler (at_sched_step)."""
    import torch
    from auratensor_b200 import synth
    from auratensor_b200.inference import SamplerConfig
    from auratensor_b200.scheduler import BatchScheduler
    assert world == 1, "the batched sampled workload runs on one GPU"
    B, n_prompt, ctx_len = args.batch, args.prompt, shape.ctx
    T, K, P, R = args.sampler
    cfgs = [SamplerConfig(T, K, P, R, 7 + b) for b in range(B)]
    total_steps = args.warmup + args.steps
    assert n_prompt + total_steps <= ctx_len, "steps exceed the context"
    keep_host = not args.no_cpu_baseline and args.layers is None
    t0 = time.time()
    model, host = build_model(shape, args.seed, ctx, world, keep_host, max_batch=B, kv_type=args.kv)
    load_s = time.time() - t0
    stream = torch.cuda.ExternalStream(model.stream())
    prompts = [synth.prompt_ids(shape, args.seed + b, n_prompt).tolist() for b in range(B)]

    def all_prompts():
        for b in range(B):
            model.forwardPromptSlot(b, prompts[b][:-1])

    prefill_dev_s, prefill_s = time_prompt(all_prompts, stream, lambda v: v)
    first = [p[-1] for p in prompts]
    start = [n_prompt - 1] * B
    hists = [list(p) for p in prompts]
    warm = model.generateSampled(first, start, args.warmup, cfgs, hists)
    first2 = [int(warm[b, -1]) for b in range(B)]
    start2 = [n_prompt - 1 + args.warmup] * B
    hists2 = [hists[b] + warm[b].tolist() for b in range(B)]
    gpus = [local]
    with ClockSampler(gpus) as clk:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = model.generateSampled(first2, start2, args.steps, cfgs, hists2)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        # e2e: the request scheduler, prompts admitted (untimed), then args.steps timed steps
        sched = BatchScheduler(model)
        ids = [sched.submit(prompts[b], total_steps + 1, cfgs[b]) for b in range(B)]
        for _ in range(args.warmup):
            sched.step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        w0 = time.perf_counter()
        for _ in range(args.steps):
            sched.step()
        w1 = time.perf_counter()
        f1.record(stream)
        f1.synchronize()
        ms_e2e = f0.elapsed_time(f1)
        sched_tokens = [sched.result(r)[0] for r in ids]
        sched.close()
    clocks = clk.summary()
    value = B * args.steps / (ms / 1000.0)
    e2e = B * args.steps / (ms_e2e / 1000.0)
    # the scheduler and the device loop are the same computation: their token streams agree
    agree = sum(int(np.array_equal(sched_tokens[b][: args.warmup + args.steps],
                                   np.concatenate([warm[b], out[b]]))) for b in range(B))
    timed_pos = [[n_prompt - 1 + args.warmup + i] * B for i in range(args.steps)]
    step_bytes = step_bytes_of(shape, world, timed_pos, B, args.kv)
    # roofline of the dominant kernel class at batch B (eager, one event pair per launch)
    tot = {}
    prof_pos = n_prompt - 1 + total_steps
    for i in range(args.profile_steps):
        p = min(prof_pos + i, ctx_len - 1)
        r = model.profileBatch([1] * B, [p] * B)
        for k, (msk, n) in r.items():
            a = tot.setdefault(k, [0.0, 0])
            a[0] += msk
            a[1] += n
    bytes_per = class_bytes(shape, world, prof_pos, B, args.kv)
    gemv = {k: v for k, v in tot.items() if k in bytes_per}
    dom = max(gemv, key=lambda k: gemv[k][0])
    avg_ms = gemv[dom][0] / max(1, gemv[dom][1])
    peak, peak_kind = load_peaks()
    achieved = bytes_per[dom] / (avg_ms / 1000.0) / 1e9
    parity = None if args.no_parity else batched_parity(shape, args.seed, ctx, B, args.sampler, args.kv)
    cpu = None
    if keep_host:
        threads = os.cpu_count() or 1
        rates = cpu_decode_sample(shape, host, threads, 4, n_prompt + 64)
        sampler_s = host_sampler_seconds(shape.vocab, args.sampler)
        v = 1.0 / (sum(1 / r for r in rates) / len(rates) + sampler_s)
        cpu = {"value": round(v, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{SAMPLE_LAYERS} of {shape.n_layers} layers + lm_head, 4 decode tokens at positions "
                         f"{n_prompt + 64}.., extrapolated to {shape.n_layers} layers, plus the host Sampler "
                         f"({sampler_s * 1e3:.3f} ms); one request at a time, as the reference's server"}
    # per step: embed; 5 per layer; lm_head, argmax (2); sample, advance
    launches_per_step = 1 + 5 * shape.n_layers + 3 + 2
    line = {
        "metric": args.metric, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args, shape), "batch": B, "requests": B, "prompt_tokens": n_prompt,
                   "context": ctx_len, "sampler": {"temperature": T, "top_k": K, "top_p": P,
                                                   "repetition_penalty": R, "seeds": [c.seed for c in cfgs]},
                   "weights": "Q8_0 (7.7 GB, > L2; no flush needed)", "parallelism": "tp1", "seed": args.seed,
                   "kv_cache": args.kv_type,
                   "step": f"one batched step = {B} tokens"},
        "e2e": {"value": round(e2e, 3), "unit": UNIT, "h2d_bytes_per_step": B * (4 + 8 + 4),
                "d2h_bytes_per_step": B * 4, "api": "at_sched_step (request scheduler)",
                "host_wall_tok_s": round(B * args.steps / (w1 - w0), 3),
                "requests_matching_device_loop": agree},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None, "bytes_per_launch": bytes_per[dom],
                     "avg_launch_us": round(avg_ms * 1000.0, 2), "step_bytes": int(step_bytes),
                     "step_frac": round(step_bytes / (ms / args.steps / 1000.0) / 1e9 / peak, 4)},
        "parity": parity,
        "kernel_ms_per_step": {k: round(v[0] / args.profile_steps, 4) for k, v in tot.items() if v[1]},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "setup": {"load_s": round(load_s, 1), "prefill_s": round(prefill_s, 2)},
        "prompt": prompt_line(shape, world, n_prompt - 1, prefill_dev_s, prefill_s, requests=B),
    }
    print(json.dumps(line), flush=True)
    finish(model, ctx, world)


def finish(model, ctx, world):
    """Releases the model (its step graphs and the peer-mapped exchange
    areas) and the context's communicator before the process group goes
    away; every rank takes the same steps."""
    import torch.distributed as dist
    from auratensor_b200 import _lib
    model.close()
    _lib.call("at_ctx_destroy", ctx)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
