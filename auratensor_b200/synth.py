"""Seeded random-init Llama-family models in GGUF block formats.

The workloads are synthetic: weights drawn from N(0, 0.02), quantized per
32-element block, norm weights 1.0 in f32, prompt ids uniform in [0, vocab).

Q4_0 quantization (one block of 32 values x): m = the value of largest
magnitude (first one on ties), d = m / -8, q = clamp(rint(x / d) + 8, 0, 15),
d stored as IEEE fp16 (round to nearest even), nibbles packed in the
reference's INTERLEAVED order: byte k = q[2k] | q[2k+1] << 4
(quant/Q4_0.java:21-22), or in llama.cpp's split-halves order (byte k =
q[k] | q[k+16] << 4) for llama.cpp-layout models. Q8_0: d = max|x| / 127,
q = rint(x / d). Q6_K (token_embd / output of llama.cpp-layout models): per
256-element block, scale_j = max|x| / 31 of each 16-element sub-block,
d = max_j scale_j / 16 (fp16; a normal number for these weights, which
Fp16.toFloat's flush-to-zero needs), int8 sc_j = rint(scale_j / d),
q = clamp(rint(x / (d sc_j)) + 32, 0, 63), packed as quant/Q6_K.java reads it.
A llama.cpp-layout model also stores its attention weights [out][in].

``numpy`` generation serves the tests (the oracle reads the same bytes);
``torch`` generation on the GPU serves large models for the benchmark, with
the same quantizer arithmetic.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .gguf import F16, F32, Q4_0, Q6_K, Q8_0, GgufWriter, U32, F32V, STR

QK = 32
QK_K = 256
LAYOUT_Q4_SPLIT_HALVES, LAYOUT_ATTN_OUT_IN = 1, 2
LAYOUT_LLAMA_CPP = LAYOUT_Q4_SPLIT_HALVES | LAYOUT_ATTN_OUT_IN


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
    layout: int = 0          # byte layout of the tensors (LAYOUT_*)
    emb_type: int = -1       # type of token_embd / output (-1: wtype)

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    def tensor_dims(self):
        """Logical dims (outer to inner) per tensor, in the reference's
        interpretation (inference/Weights.java:84-112)."""
        d, f, hd = self.dim, self.ffn, self.head_dim
        et = self.wtype if self.emb_type < 0 else self.emb_type
        oi = bool(self.layout & LAYOUT_ATTN_OUT_IN)  # attention bytes [out][in] (llama.cpp)

        def att(din, dout):
            return (dout, din) if oi else (din, dout)

        out = [("token_embd.weight", (self.vocab, d), et)]
        for L in range(self.n_layers):
            p = f"blk.{L}."
            out += [
                (p + "attn_q.weight", att(d, self.n_heads * hd), self.wtype),
                (p + "attn_k.weight", att(d, self.n_kv_heads * hd), self.wtype),
                (p + "attn_v.weight", att(d, self.n_kv_heads * hd), self.wtype),
                (p + "attn_output.weight", att(self.n_heads * hd, d), self.wtype),
                (p + "ffn_gate.weight", (f, d), self.wtype),
                (p + "ffn_up.weight", (f, d), self.wtype),
                (p + "ffn_down.weight", (d, f), self.wtype),
                (p + "attn_norm.weight", (d,), F32),
                (p + "ffn_norm.weight", (d,), F32),
            ]
        out.append(("output_norm.weight", (d,), F32))
        out.append(("output.weight", (self.vocab, d), et))
        return out

    def weight_bytes(self) -> int:
        tot = 0
        for name, dims, t in self.tensor_dims():
            n = int(np.prod(dims))
            tot += n * 4 if t == F32 else ((n // QK_K) * 210 if t == Q6_K else (n // QK) * (18 if t == Q4_0 else 34))
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
# llama.cpp-layout small model: split-halves Q4_0 nibbles, [out][in] attention, Q6_K embedding and output
TINY_LLAMACPP = ModelShape("tiny-llamacpp", 2, 256, 512, 4, 2, 1000, 10000.0, 64, Q4_0,
                           layout=LAYOUT_LLAMA_CPP, emb_type=Q6_K)


# --------------------------------------------------------------------------
# numpy quantizers
# --------------------------------------------------------------------------
def quantize_q4_0(x: np.ndarray, split: bool = False) -> np.ndarray:
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
    out[:, 2:] = (q[:, :16] | (q[:, 16:] << 4)) if split else (q[:, 0::2] | (q[:, 1::2] << 4))
    return out.reshape(-1)


def _fp16_ftz(d16: np.ndarray) -> np.ndarray:
    """fp16 -> float32 with subnormals flushed (Fp16.toFloat)."""
    f = d16.astype(np.float32)
    return np.where((d16.view(np.uint16) & 0x7C00) == 0, np.float32(0.0), f).astype(np.float32)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    xb = np.asarray(x, dtype=np.float32).reshape(-1, QK_K)
    nb = xb.shape[0]
    sub = xb.reshape(nb, 16, 16)
    sreal = np.abs(sub).max(axis=2) / np.float32(31.0)
    # d = max scale / 16 (int8 scales up to 16) keeps d a normal fp16 for
    # N(0, 0.02) weights: Fp16.toFloat flushes subnormal scales to zero
    d16 = (sreal.max(axis=1) / np.float32(16.0)).astype(np.float16)
    d = _fp16_ftz(d16)
    safe = np.where(d == 0, np.float32(1.0), d)
    sc = np.where(d[:, None] == 0, 0, np.clip(np.rint(sreal / safe[:, None]), -128, 127)).astype(np.int8)
    eff = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
    effs = np.where(eff == 0, np.float32(1.0), eff)
    q = np.where(eff[:, :, None] == 0, 32, np.clip(np.rint(sub / effs[:, :, None]) + 32, 0, 63))
    q = q.astype(np.int32).reshape(nb, 2, 4, 32)  # [half n][group j][l]
    ql = np.empty((nb, 2, 64), dtype=np.uint8)
    for jj in range(2):
        ql[:, :, 32 * jj:32 * jj + 32] = ((q[:, :, jj, :] & 0xF) | ((q[:, :, jj + 2, :] & 0xF) << 4)).astype(np.uint8)
    qh = np.zeros((nb, 2, 32), dtype=np.int32)
    for j in range(4):
        qh |= ((q[:, :, j, :] >> 4) & 3) << (2 * j)
    out = np.empty((nb, 210), dtype=np.uint8)
    out[:, :128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.astype(np.uint8).reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(nb, 2)
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


def quantize(x: np.ndarray, wtype: int, layout: int = 0) -> np.ndarray:
    if wtype == Q4_0:
        return quantize_q4_0(x, split=bool(layout & LAYOUT_Q4_SPLIT_HALVES))
    if wtype == Q8_0:
        return quantize_q8_0(x)
    if wtype == Q6_K:
        return quantize_q6_k(x)
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
                chunks.append(quantize((rng.standard_normal(c, dtype=np.float32) * np.float32(std)), t, shape.layout))
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
def quantize_q6_k_torch(x):
    """quantize_q6_k on the device (same arithmetic)."""
    import torch
    xb = x.reshape(-1, QK_K).float()
    nb = xb.shape[0]
    sub = xb.reshape(nb, 16, 16)
    sreal = sub.abs().amax(dim=2) / 31.0
    d16 = (sreal.amax(dim=1) / 16.0).to(torch.float16)
    d = torch.where((d16.view(torch.int16) & 0x7C00) == 0, torch.zeros_like(d16, dtype=torch.float32), d16.float())
    safe = torch.where(d == 0, torch.ones_like(d), d)
    sc = torch.where((d == 0)[:, None], torch.zeros_like(sreal), torch.round(sreal / safe[:, None]).clamp_(-128, 127))
    eff = d[:, None] * sc
    effs = torch.where(eff == 0, torch.ones_like(eff), eff)
    q = torch.where((eff == 0)[:, :, None], torch.full_like(sub, 32.0),
                    (torch.round(sub / effs[:, :, None]) + 32).clamp_(0, 63))
    q = q.to(torch.int32).reshape(nb, 2, 4, 32)
    out = torch.empty((nb, 210), dtype=torch.uint8, device=x.device)
    ql = torch.cat([(q[:, :, jj, :] & 0xF) | ((q[:, :, jj + 2, :] & 0xF) << 4) for jj in range(2)], dim=2)
    qh = torch.zeros((nb, 2, 32), dtype=torch.int32, device=x.device)
    for j in range(4):
        qh |= ((q[:, :, j, :] >> 4) & 3) << (2 * j)
    out[:, :128] = ql.reshape(nb, 128).to(torch.uint8)
    out[:, 128:192] = qh.reshape(nb, 64).to(torch.uint8)
    out[:, 192:208] = sc.to(torch.int8).view(torch.uint8)
    out[:, 208:210] = d16.view(torch.uint8).view(nb, 2)
    return out.reshape(-1)


def quantize_torch(x, wtype: int, layout: int = 0):
    import torch
    if wtype == Q6_K:
        return quantize_q6_k_torch(x)
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
        if layout & LAYOUT_Q4_SPLIT_HALVES:
            out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
        else:
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


def generate_torch_tensor(dims, wtype: int, gen, device, std: float = 0.02, layout: int = 0):
    """One quantized tensor generated on the device, chunked to bound memory."""
    import torch
    n = int(np.prod(dims))
    if wtype == F32:
        return torch.ones(n, dtype=torch.float32, device=device).view(torch.uint8)
    per, bpb = (QK_K, 210) if wtype == Q6_K else (QK, 18 if wtype == Q4_0 else 34)
    out = torch.empty((n // per) * bpb, dtype=torch.uint8, device=device)
    step = 1 << 26
    for s in range(0, n, step):
        c = min(step, n - s)
        x = torch.randn(c, generator=gen, device=device, dtype=torch.float32) * std
        out[(s // per) * bpb:((s + c) // per) * bpb] = quantize_torch(x, wtype, layout)
    return out
