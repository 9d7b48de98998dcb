"""Seeded random-init Llama-family models in GGUF block formats.

The workloads are synthetic: weights drawn from N(0, 0.02), quantized per
32-element block, norm weights 1.0 in f32, prompt ids uniform in [0, vocab).

Q4_0 quantization (one block of 32 values x): m = the value of largest
magnitude (first one on ties), d = m / -8, q = clamp(rint(x / d) + 8, 0, 15),
d stored as IEEE fp16 (round to nearest even), nibbles packed in the
reference's INTERLEAVED order: byte k = q[2k] | q[2k+1] << 4
(quant/Q4_0.java:21-22). Q8_0: d = max|x| / 127, q = rint(x / d).

``numpy`` generation serves the tests (the oracle reads the same bytes);
``torch`` generation on the GPU serves large models for the benchmark, with
the same quantizer arithmetic.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .gguf import F16, F32, Q4_0, Q8_0, GgufWriter, U32, F32V, STR

QK = 32


@dataclass(frozen=True)
class ModelShape:
    name: str
    n_layers: int
    dim: int
    ffn: int
    n_heads: int
    n_kv_heads: int
    vocab: int
    rope_theta: float
    ctx: int
    wtype: int = Q4_0
    tied: bool = False
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def tensor_dims(self):
        """Logical dims (outer to inner) per tensor, in the reference's
        interpretation (inference/Weights.java:84-112)."""
        d, f, hd = self.dim, self.ffn, self.head_dim
        out = [("token_embd.weight", (self.vocab, d), self.wtype)]
        for L in range(self.n_layers):
            p = f"blk.{L}."
            out += [
                (p + "attn_q.weight", (d, self.n_heads * hd), self.wtype),
                (p + "attn_k.weight", (d, self.n_kv_heads * hd), self.wtype),
                (p + "attn_v.weight", (d, self.n_kv_heads * hd), self.wtype),
                (p + "attn_output.weight", (self.n_heads * hd, d), self.wtype),
                (p + "ffn_gate.weight", (f, d), self.wtype),
                (p + "ffn_up.weight", (f, d), self.wtype),
                (p + "ffn_down.weight", (d, f), self.wtype),
                (p + "attn_norm.weight", (d,), F32),
                (p + "ffn_norm.weight", (d,), F32),
            ]
        out.append(("output_norm.weight", (d,), F32))
        out.append(("output.weight", (self.vocab, d), self.wtype))
        return out

    def weight_bytes(self) -> int:
        tot = 0
        for name, dims, t in self.tensor_dims():
            n = int(np.prod(dims))
            tot += n * 4 if t == F32 else (n // QK) * (18 if t == Q4_0 else 34)
        return tot

    def metadata(self):
        return [
            ("general.architecture", STR, "llama"),
            ("llama.context_length", U32, self.ctx),
            ("llama.embedding_length", U32, self.dim),
            ("llama.block_count", U32, self.n_layers),
            ("llama.attention.head_count", U32, self.n_heads),
            ("llama.attention.head_count_kv", U32, self.n_kv_heads),
            ("llama.feed_forward_length", U32, self.ffn),
            ("llama.rope.freq_base", F32V, float(self.rope_theta)),
            ("llama.attention.layer_norm_rms_epsilon", F32V, float(self.eps)),
            ("llama.vocab_size", U32, self.vocab),
        ]


# The model shapes of the benchmark workloads.
LLAMA32_1B = ModelShape("llama-3.2-1b", 16, 2048, 8192, 32, 8, 128256, 500000.0, 128, Q4_0, tied=True)
LLAMA3_8B = ModelShape("llama-3-8b", 32, 4096, 14336, 32, 8, 128256, 500000.0, 2048, Q4_0)
MISTRAL_7B = ModelShape("mistral-7b", 32, 4096, 14336, 32, 8, 32000, 1e6, 4096, Q8_0)
LLAMA3_70B = ModelShape("llama-3-70b", 80, 8192, 28672, 64, 8, 128256, 500000.0, 8192, Q4_0)
# Small shapes for parity tests.
TINY = ModelShape("tiny", 2, 256, 512, 4, 2, 1000, 10000.0, 64, Q4_0)
TINY_Q8 = ModelShape("tiny-q8", 2, 256, 512, 4, 2, 1000, 1e6, 64, Q8_0)


# --------------------------------------------------------------------------
# numpy quantizers
# --------------------------------------------------------------------------
def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    xb = np.asarray(x, dtype=np.float32).reshape(-1, QK)
    nb = xb.shape[0]
    idx = np.argmax(np.abs(xb), axis=1)
    m = xb[np.arange(nb), idx]
    d = (m / np.float32(-8.0)).astype(np.float32)
    safe = np.where(d == 0, np.float32(1.0), d).astype(np.float32)
    q = np.rint(xb / safe[:, None]) + 8
    q = np.where(d[:, None] == 0, 8, q)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.empty((nb, 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q[:, 0::2] | (q[:, 1::2] << 4)
    return out.reshape(-1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    xb = np.asarray(x, dtype=np.float32).reshape(-1, QK)
    nb = xb.shape[0]
    amax = np.max(np.abs(xb), axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    safe = np.where(d == 0, np.float32(1.0), d).astype(np.float32)
    q = np.clip(np.rint(xb / safe[:, None]), -127, 127).astype(np.int8)
    q = np.where(d[:, None] == 0, 0, q).astype(np.int8)
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize(x: np.ndarray, wtype: int) -> np.ndarray:
    if wtype == Q4_0:
        return quantize_q4_0(x)
    if wtype == Q8_0:
        return quantize_q8_0(x)
    if wtype == F32:
        return np.asarray(x, dtype=np.float32).view(np.uint8).reshape(-1)
    if wtype == F16:
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(-1)
    raise ValueError(wtype)


def generate_numpy(shape: ModelShape, seed: int, std: float = 0.02) -> dict:
    """{name: {"type", "dims", "data" (uint8 array)}} in a fixed name order."""
    rng = np.random.default_rng(seed)
    tensors = {}
    for name, dims, t in shape.tensor_dims():
        n = int(np.prod(dims))
        if t == F32:
            data = np.ones(n, dtype=np.float32).view(np.uint8)
        elif shape.tied and name == "output.weight":
            data = tensors["token_embd.weight"]["data"].copy()
        else:
            chunks = []
            step = 1 << 24
            for s in range(0, n, step):
                c = min(step, n - s)
                chunks.append(quantize((rng.standard_normal(c, dtype=np.float32) * np.float32(std)), t))
            data = np.concatenate(chunks)
        tensors[name] = {"type": t, "dims": dims, "data": data}
    return tensors


def prompt_ids(shape: ModelShape, seed: int, n: int) -> np.ndarray:
    return np.random.default_rng(seed + 1).integers(0, shape.vocab, size=n, dtype=np.int64)


def write_gguf(shape: ModelShape, tensors: dict, path: str) -> None:
    w = GgufWriter()
    for k, vt, v in shape.metadata():
        w.add_kv(k, vt, v)
    for name, dims, t in shape.tensor_dims():
        if name in tensors:
            w.add_tensor(name, dims, tensors[name]["type"], np.ascontiguousarray(tensors[name]["data"]))
    w.write(path)


# --------------------------------------------------------------------------
# torch (GPU) quantizers: same arithmetic, for multi-GB models
# --------------------------------------------------------------------------
def quantize_torch(x, wtype: int):
    import torch
    xb = x.reshape(-1, QK).float()
    nb = xb.shape[0]
    if wtype == Q4_0:
        idx = xb.abs().argmax(dim=1, keepdim=True)
        m = xb.gather(1, idx).squeeze(1)
        d = m / -8.0
        safe = torch.where(d == 0, torch.ones_like(d), d)
        q = torch.round(xb / safe[:, None]) + 8
        q = torch.where((d == 0)[:, None], torch.full_like(q, 8), q).clamp_(0, 15).to(torch.uint8)
        out = torch.empty((nb, 18), dtype=torch.uint8, device=x.device)
        out[:, 0:2] = d.to(torch.float16).view(torch.uint8).view(nb, 2)
        out[:, 2:] = q[:, 0::2] | (q[:, 1::2] << 4)
    elif wtype == Q8_0:
        amax = xb.abs().amax(dim=1)
        d = amax / 127.0
        safe = torch.where(d == 0, torch.ones_like(d), d)
        q = torch.round(xb / safe[:, None]).clamp_(-127, 127)
        q = torch.where((d == 0)[:, None], torch.zeros_like(q), q).to(torch.int8)
        out = torch.empty((nb, 34), dtype=torch.uint8, device=x.device)
        out[:, 0:2] = d.to(torch.float16).view(torch.uint8).view(nb, 2)
        out[:, 2:] = q.view(torch.uint8)
    else:
        raise ValueError(wtype)
    return out.reshape(-1)


def generate_torch_tensor(dims, wtype: int, gen, device, std: float = 0.02):
    """One quantized tensor generated on the device, chunked to bound memory."""
    import torch
    n = int(np.prod(dims))
    if wtype == F32:
        return torch.ones(n, dtype=torch.float32, device=device).view(torch.uint8)
    bpb = 18 if wtype == Q4_0 else 34
    out = torch.empty((n // QK) * bpb, dtype=torch.uint8, device=device)
    step = 1 << 26
    for s in range(0, n, step):
        c = min(step, n - s)
        x = torch.randn(c, generator=gen, device=device, dtype=torch.float32) * std
        out[(s // QK) * bpb:((s + c) // QK) * bpb] = quantize_torch(x, wtype)
    return out
