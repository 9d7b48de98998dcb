"""Builds libauratensor_cuda.so in-tree with nvcc for sm_100a.

Objects go to ``auratensor_b200/_build/``; the shared library to
``auratensor_b200/lib/libauratensor_cuda.so``. Translation units compile in
parallel and are rebuilt only when a source or header is newer than the
object.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libauratensor_cuda.so")
SOURCES = ["at_runtime.cu", "gemv.cu", "gemm_tc.cu", "prompt_attn_tc.cu", "model.cu", "decode_step.cu", "q6k.cu", "sample.cu", "sampler.cpp", "sched.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "auratensor.h"))
    return hs


def _compile(src: str, verbose: bool, ptxas_v: bool) -> str:
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD, src + ".o")
    newest = max([os.path.getmtime(path)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest and not ptxas_v:
        return obj
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-O3",
           "-I", os.path.join(ROOT, "include"), "-c", path, "-o", obj]
    if src.endswith(".cu"):
        cmd[1:1] = ["--expt-relaxed-constexpr"]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
    else:
        cmd = [nvcc(), "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-I", os.path.join(ROOT, "include"),
               "-c", path, "-o", obj]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if ptxas_v:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    with cf.ThreadPoolExecutor(max_workers=len(srcs)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_v), srcs))
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs):
        return LIB
    cmd = [nvcc(), "-shared", *ARCH, "-Xcompiler", "-fPIC", "-o", LIB + ".tmp", *objs, "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_v="--ptxas" in sys.argv))
