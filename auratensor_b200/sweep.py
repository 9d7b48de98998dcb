"""Fused-dequant GEMV sweep: device time per call and effective bandwidth.

Each shape is timed as a CUDA graph of back-to-back ``at_gemv`` calls that
cycle over enough copies of the matrix to exceed the 126 MB L2, so every
call streams its weights from HBM. Output: one JSON line per case with the
time per call (µs) and the algorithmic bytes (weights + x + y) per second.

    python -m auratensor_b200.sweep                         # Q4_0/Q8_0, batch 1 and 8
    python -m auratensor_b200.sweep --types q4_0 --batch 1
    python -m auratensor_b200.sweep --one 14336 4096 N q4_0 --calls 8   # a few eager calls (for ncu)
    python -m auratensor_b200.sweep --one 14336 4096 N q8_0 --batch 8  # the same at batch 8
    python -m auratensor_b200.sweep --gemm --types q4_0             # tensor-core prompt GEMM, TFLOP/s

Shapes are (rows, cols) of the stored matrix: orientation N computes
y[rows] = W x[cols] (ffn, lm_head), orientation T computes y[cols] = W^T x[rows]
(the attention projections of inference/LlamaModel.java:205-236, stored [in][out]).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import synth
from .quant import ORIENT_N, ORIENT_T, QMatrix

Q4_0, Q8_0 = 2, 8
TYPES = {"q4_0": Q4_0, "q8_0": Q8_0}
# Llama-3-8B projections and the square 2048 case (rows, cols, orientation)
SHAPES = [
    (2048, 2048, ORIENT_N), (8192, 2048, ORIENT_N), (2048, 8192, ORIENT_N),
    (14336, 4096, ORIENT_N), (4096, 14336, ORIENT_N), (128256, 4096, ORIENT_N),
    (4096, 6144, ORIENT_T), (4096, 4096, ORIENT_T),
]
L2_BYTES = 126 << 20


def block_bytes(qt: int) -> int:
    return 18 if qt == Q4_0 else 34


def time_case(qt: int, rows: int, cols: int, orient: int, batch: int, dev: torch.device, reps: int = 4) -> dict:
    g = torch.Generator(device=dev).manual_seed(rows * 31 + cols)
    nbytes = rows * cols // 32 * block_bytes(qt)
    ncopy = max(2, -(-(3 * L2_BYTES) // nbytes))
    mats = [QMatrix(qt, orient, rows, cols, synth.generate_torch_tensor((rows, cols), qt, g, dev))
            for _ in range(ncopy)]
    n_in, n_out = (cols, rows) if orient == ORIENT_N else (rows, cols)
    x = torch.randn((batch, n_in), device=dev)
    y = torch.empty((batch, n_out), device=dev)
    for m in mats:
        m.gemv(x, y)
    torch.cuda.synchronize()
    calls = reps * ncopy
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(calls):
                mats[i % ncopy].gemv(x, y)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / calls
    algo = nbytes + batch * (n_in + n_out) * 4
    del graph, mats
    torch.cuda.empty_cache()
    return {"type": "q4_0" if qt == Q4_0 else "q8_0", "rows": rows, "cols": cols,
            "orient": "N" if orient == ORIENT_N else "T", "batch": batch, "us_per_call": round(us, 2),
            "GBps": round(algo / us / 1e3, 1), "weight_bytes": nbytes}


# Llama-3-8B prompt projections (rows, cols, orientation) for the tensor-core GEMM
GEMM_SHAPES = [(4096, 6144, ORIENT_T), (4096, 4096, ORIENT_T), (14336, 4096, ORIENT_N), (4096, 14336, ORIENT_N)]


def time_gemm(qt: int, rows: int, cols: int, orient: int, tokens: int, dev: torch.device, reps: int = 10) -> dict:
    """Device time of one at_gemm_tc call (bf16 conversion of x + the tcgen05 GEMM)."""
    g = torch.Generator(device=dev).manual_seed(rows + cols)
    m = QMatrix(qt, orient, rows, cols, synth.generate_torch_tensor((rows, cols), qt, g, dev))
    n_in, n_out = (cols, rows) if orient == ORIENT_N else (rows, cols)
    x = torch.randn((tokens, n_in), device=dev)
    y = torch.empty((tokens, n_out), device=dev)
    m.gemm(x, y)
    times = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        m.gemm(x, y)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1000.0)
    us = sorted(times)[len(times) // 2]
    flops = 2.0 * n_in * n_out * tokens
    return {"type": "q4_0" if qt == Q4_0 else "q8_0", "rows": rows, "cols": cols,
            "orient": "N" if orient == ORIENT_N else "T", "tokens": tokens, "us_per_call": round(us, 2),
            "TFLOPs": round(flops / us / 1e6, 1)}


def run_one(rows: int, cols: int, orient: int, qt: int, calls: int, dev: torch.device, batch: int = 1) -> None:
    """A few eager calls on 4 copies of one matrix (a small case for ncu)."""
    g = torch.Generator(device=dev).manual_seed(0)
    mats = [QMatrix(qt, orient, rows, cols, synth.generate_torch_tensor((rows, cols), qt, g, dev))
            for _ in range(4)]
    x = torch.randn((batch, cols if orient == ORIENT_N else rows), device=dev)
    for i in range(calls):
        mats[i % 4].gemv(x)
    torch.cuda.synchronize()
    print(json.dumps({"calls": calls, "rows": rows, "cols": cols}))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--types", default="q4_0,q8_0")
    ap.add_argument("--batch", default="1,8")
    ap.add_argument("--one", nargs=4, metavar=("ROWS", "COLS", "N|T", "TYPE"))
    ap.add_argument("--calls", type=int, default=8)
    ap.add_argument("--gemm", action="store_true", help="time the tensor-core prompt GEMM instead")
    ap.add_argument("--tokens", default="128,512")
    args = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    if args.gemm:
        for t in args.types.split(","):
            for rows, cols, orient in GEMM_SHAPES:
                for n in (int(v) for v in args.tokens.split(",")):
                    print(json.dumps(time_gemm(TYPES[t.lower()], rows, cols, orient, n, dev)), flush=True)
        return
    if args.one:
        rows, cols, o, t = args.one
        run_one(int(rows), int(cols), ORIENT_N if o.upper() == "N" else ORIENT_T, TYPES[t.lower()], args.calls, dev,
                int(args.batch.split(",")[0]))
        return
    for t in args.types.split(","):
        for rows, cols, orient in SHAPES:
            for b in (int(v) for v in args.batch.split(",")):
                print(json.dumps(time_case(TYPES[t.lower()], rows, cols, orient, b, dev)), flush=True)


if __name__ == "__main__":
    main()
