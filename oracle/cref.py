"""ctypes wrapper of oracle/ref_decode.c (test infrastructure and CPU baseline only).

The shared object is built per host CPU model (``-march=native``) into
``oracle/_build/`` by ``oracle/Makefile``.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class RdCfg(C.Structure):
    _fields_ = [("dim", C.c_int), ("ffn", C.c_int), ("n_heads", C.c_int), ("n_kv", C.c_int), ("vocab", C.c_int),
                ("ctx", C.c_int), ("n_layers", C.c_int), ("rope_base", C.c_float), ("eps", C.c_float),
                ("layout", C.c_int), ("kv_q8", C.c_int)]


def host_tag() -> str:
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith(("model name", "flags")):
                    model += line
    except OSError:
        pass
    return hashlib.sha1(model.encode()).hexdigest()[:10]


def build() -> str:
    tag = host_tag()
    subprocess.run(["make", "-s", "-C", HERE, f"HOSTTAG={tag}"], check=True)
    return os.path.join(HERE, "_build", f"libref_decode-{tag}.so")


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(build())
        L.rd_create.restype = C.c_void_p
        L.rd_create.argtypes = [C.POINTER(RdCfg), C.c_int]
        L.rd_set_tensor.restype = C.c_int
        L.rd_set_tensor.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
        L.rd_forward_step.restype = C.POINTER(C.c_float)
        L.rd_forward_step.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.rd_forward_layers.restype = None
        L.rd_forward_layers.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.rd_kv.restype = None
        L.rd_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.rd_times.argtypes = [C.c_void_p] + [C.POINTER(C.c_double)] * 3
        L.rd_destroy.argtypes = [C.c_void_p]
        _lib = L
    return _lib


class RefDecoder:
    """The reference's decode path in C: load-time dequant, FP32 sgemv."""

    def __init__(self, shape, n_layers: int | None = None, threads: int = 1, kv_type: int = 0):
        """kv_type 8: K/V rounded as the device's Q8_0 KV cache stores them."""
        self.shape = shape
        self.n_layers = shape.n_layers if n_layers is None else n_layers
        cfg = RdCfg(shape.dim, shape.ffn, shape.n_heads, shape.n_kv_heads, shape.vocab, shape.ctx, self.n_layers,
                    float(shape.rope_theta), float(shape.eps), int(getattr(shape, "layout", 0)), int(kv_type == 8))
        self._h = lib().rd_create(C.byref(cfg), threads)
        self._keep = []

    def set_tensor(self, name: str, ggml_type: int, data, numel: int) -> None:
        arr = np.ascontiguousarray(np.frombuffer(memoryview(data), dtype=np.uint8))
        self._keep.append(arr)  # token_embd is referenced, not copied
        if lib().rd_set_tensor(self._h, name.encode(), ggml_type, arr.ctypes.data_as(C.c_void_p), numel) != 0:
            raise ValueError(f"ref decoder rejected {name}")

    def forward_step(self, token: int, pos: int) -> np.ndarray:
        p = lib().rd_forward_step(self._h, int(token), int(pos))
        return np.ctypeslib.as_array(p, shape=(self.shape.vocab,)).copy()

    def forward_layers(self, token: int, pos: int) -> None:
        """forward_step without the lm_head: fills the KV cache only."""
        lib().rd_forward_layers(self._h, int(token), int(pos))

    def kv(self, layer: int, kv_head: int, pos: int):
        hd = self.shape.dim // self.shape.n_heads
        k = np.empty(hd, dtype=np.float32)
        v = np.empty(hd, dtype=np.float32)
        lib().rd_kv(self._h, layer, kv_head, pos, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p))
        return k, v

    def times(self):
        a, b, c = C.c_double(), C.c_double(), C.c_double()
        lib().rd_times(self._h, C.byref(a), C.byref(b), C.byref(c))
        return a.value, b.value, c.value

    def close(self):
        if self._h:
            lib().rd_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
