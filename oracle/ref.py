"""Numpy restatement of the reference decode path (test infrastructure only).

Every function names the reference file and lines it restates (paths are
relative to the AuraTensor source tree, ``src/main/java/io/auratensor/``).
The restatement follows the reference's ALGORITHM exactly: quantized tensors
are dequantized to FP32 once at load (inference/Weights.java:185-203) and
every projection is an FP32 matrix-vector product (core/Kernels.java:350-371).
Only the floating-point summation order differs from the Java SIMD lanes
(numpy/BLAS order), which is below the parity tolerances used by the tests.

This module is the ORACLE: only tests, ``__graft_entry__.smoke()`` and the
CPU-baseline legs of ``bench.py`` may use it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .java_random import JavaRandom

QK = 32                 # quant/QuantBlock.java:27 BLOCK_SIZE
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q6_K = 0, 1, 2, 8, 14   # format/GgufTensorType.java:15-27
BLOCK_BYTES = {GGML_Q4_0: 18, GGML_Q8_0: 34, GGML_Q6_K: 210}           # quant/QuantBlock.java:34-39, quant/Q6_K.java:41
QK_K = 256
# Byte layouts: 0 = the reference's (interleaved Q4_0 nibbles, attention
# weights read [in][out]); llama.cpp exports use split-halves nibbles (bit 0)
# and [out][in] attention weights (bit 1). The reference reads only the first.
LAYOUT_Q4_SPLIT_HALVES, LAYOUT_ATTN_OUT_IN = 1, 2
LAYOUT_LLAMA_CPP = LAYOUT_Q4_SPLIT_HALVES | LAYOUT_ATTN_OUT_IN


# --------------------------------------------------------------------------
# fp16 decode with flush-to-zero: core/Fp16.java:19-37
# --------------------------------------------------------------------------
def fp16_bits_to_f32(bits) -> np.ndarray:
    """Fp16.toFloat: subnormal -> signed zero, inf/nan kept, normal rebias."""
    h = np.asarray(bits, dtype=np.uint16).astype(np.uint32)
    s = (h >> 15) & 1
    e = (h >> 10) & 0x1F
    m = h & 0x3FF
    normal = (s << 31) | ((e + 112) << 23) | (m << 13)
    zero = s << 31
    inf = (s << 31) | 0x7F800000
    out = np.where(e == 0, zero, np.where(e == 0x1F, np.where(m == 0, inf, 0x7FC00000), normal))
    return out.astype(np.uint32).view(np.float32)


# --------------------------------------------------------------------------
# Block codecs: quant/Q4_0.java:32-45, quant/Q8_0.java:32-44
# --------------------------------------------------------------------------
def q4_0_dequant(blocks, n: int) -> np.ndarray:
    """Q4_0.dequantToFloat: w[32b+2k] = (lo(qs[k])-8)*d, w[32b+2k+1] = (hi(qs[k])-8)*d."""
    nb = n // QK
    raw = np.frombuffer(memoryview(blocks), dtype=np.uint8, count=nb * 18).reshape(nb, 18)
    d = fp16_bits_to_f32(raw[:, 0].astype(np.uint16) | (raw[:, 1].astype(np.uint16) << 8))
    qs = raw[:, 2:]
    q = np.empty((nb, QK), dtype=np.int8)
    q[:, 0::2] = (qs & 0x0F).astype(np.int8) - 8
    q[:, 1::2] = (qs >> 4).astype(np.int8) - 8
    return (q.astype(np.float32) * d[:, None]).reshape(-1)


def q4_0_dequant_split(blocks, n: int) -> np.ndarray:
    """Q4_0 in llama.cpp's nibble order (not the reference's): element k of a
    block is the low nibble of qs[k], element k + 16 its high nibble."""
    nb = n // QK
    raw = np.frombuffer(memoryview(blocks), dtype=np.uint8, count=nb * 18).reshape(nb, 18)
    d = fp16_bits_to_f32(raw[:, 0].astype(np.uint16) | (raw[:, 1].astype(np.uint16) << 8))
    qs = raw[:, 2:]
    q = np.empty((nb, QK), dtype=np.int8)
    q[:, :16] = (qs & 0x0F).astype(np.int8) - 8
    q[:, 16:] = (qs >> 4).astype(np.int8) - 8
    return (q.astype(np.float32) * d[:, None]).reshape(-1)


def q6_k_dequant(blocks, n: int) -> np.ndarray:
    """Q6_K.dequantToFloat (quant/Q6_K.java:54-102), the published llama.cpp
    dequantize_row_q6_K: per 210-byte block of 256 elements, ql[128] low
    nibbles, qh[64] high 2-bit pairs, int8 scales[16], fp16 d (flush-to-zero);
    y[n + l + 32 j] = (d * scale[n/16 + l/16 + 2 j]) * (q - 32) for the two
    halves n = 0, 128, l = 0..31, j = 0..3, in float."""
    nb = n // QK_K
    raw = np.frombuffer(memoryview(blocks), dtype=np.uint8, count=nb * 210).reshape(nb, 210)
    d = fp16_bits_to_f32(raw[:, 208].astype(np.uint16) | (raw[:, 209].astype(np.uint16) << 8))
    sc = raw[:, 192:208].view(np.int8).astype(np.float32)
    y = np.empty((nb, QK_K), dtype=np.float32)
    l = np.arange(32)
    for half in range(2):
        ql = raw[:, 64 * half: 64 * half + 64].astype(np.int32)
        qh = raw[:, 128 + 32 * half: 128 + 32 * half + 32].astype(np.int32)
        lo, hi = ql[:, l], ql[:, l + 32]
        qs = [(lo & 0xF) | (((qh >> 0) & 3) << 4), (hi & 0xF) | (((qh >> 2) & 3) << 4),
              ((lo >> 4) & 0xF) | (((qh >> 4) & 3) << 4), ((hi >> 4) & 0xF) | (((qh >> 6) & 3) << 4)]
        for j in range(4):
            s_ = sc[:, 8 * half + l // 16 + 2 * j]
            y[:, 128 * half + 32 * j + l] = (d[:, None] * s_) * (qs[j] - 32).astype(np.float32)
    return y.reshape(-1)


def q8_0_dequant(blocks, n: int) -> np.ndarray:
    """Q8_0.dequantToFloat: w[32b+i] = int8(qs[i]) * d."""
    nb = n // QK
    raw = np.frombuffer(memoryview(blocks), dtype=np.uint8, count=nb * 34).reshape(nb, 34)
    d = fp16_bits_to_f32(raw[:, 0].astype(np.uint16) | (raw[:, 1].astype(np.uint16) << 8))
    q = raw[:, 2:].view(np.int8).astype(np.float32)
    return (q * d[:, None]).reshape(-1)


def dequant(ggml_type: int, data, n: int, layout: int = 0) -> np.ndarray:
    """Load-time conversion of one tensor to FP32 (inference/Weights.java:167-216)."""
    if ggml_type == GGML_F32:
        return np.frombuffer(memoryview(data), dtype=np.float32, count=n).copy()
    if ggml_type == GGML_F16:
        return fp16_bits_to_f32(np.frombuffer(memoryview(data), dtype=np.uint16, count=n))
    if ggml_type == GGML_Q4_0:
        return q4_0_dequant_split(data, n) if layout & LAYOUT_Q4_SPLIT_HALVES else q4_0_dequant(data, n)
    if ggml_type == GGML_Q8_0:
        return q8_0_dequant(data, n)
    if ggml_type == GGML_Q6_K:
        return q6_k_dequant(data, n)
    raise ValueError(f"unsupported type {ggml_type}")


def q_dot(ggml_type: int, blocks, x: np.ndarray) -> np.float32:
    """Row dot with dequantToFloat semantics (the semantics the model uses).

    Q4_0.dot / Q8_0.dot (quant/Q4_0.java:51-90, quant/Q8_0.java:54-93) depend
    on the SIMD lane width and cover only part of each block below 512-bit
    vectors; the oracle therefore defines dot as dequantToFloat followed by an
    FP32 dot, which is what LlamaModel effectively computes.
    """
    w = dequant(ggml_type, blocks, x.size)
    return np.float32(np.dot(w, x.astype(np.float32)))


# --------------------------------------------------------------------------
# Kernels: core/Kernels.java
# --------------------------------------------------------------------------
def sgemv(A: np.ndarray, x: np.ndarray) -> np.ndarray:
    """Kernels.sgemv (core/Kernels.java:350-371): y[M] = A[M,K] x[K], fp32."""
    return (A.astype(np.float32, copy=False) @ x.astype(np.float32, copy=False)).astype(np.float32)


def sgemm(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Kernels.sgemm (core/Kernels.java:395-452): C = A B, fp32."""
    return (A.astype(np.float32) @ B.astype(np.float32)).astype(np.float32)


def rmsnorm_inplace(x: np.ndarray, w: np.ndarray, eps: float) -> None:
    """Kernels.rmsNormInPlace (core/Kernels.java:100-154).

    invRms = (float)(1.0 / Math.sqrt(sumSq / (float) d + eps)) with the
    division and the eps add in float, sqrt and reciprocal in double;
    out = (x * invRms) * gamma in float.
    """
    d = x.shape[-1]
    rows = x.reshape(-1, d)
    for r in range(rows.shape[0]):
        v = rows[r]
        sum_sq = np.float32(np.dot(v, v))
        mean = np.float32(np.float32(sum_sq / np.float32(d)) + np.float32(eps))
        inv = np.float32(1.0 / math.sqrt(float(mean)))
        rows[r] = (v * inv).astype(np.float32) * w.astype(np.float32)


def softmax_inplace(x: np.ndarray, n: int | None = None) -> None:
    """Kernels.softmaxInPlaceSegment (core/Kernels.java:181-232) on x[:n]."""
    n = x.shape[-1] if n is None else n
    seg = x[..., :n]
    mx = np.max(seg, axis=-1, keepdims=True).astype(np.float32)
    e = np.exp((seg - mx).astype(np.float64)).astype(np.float32)
    s = np.sum(e, axis=-1, keepdims=True, dtype=np.float32)
    inv = (np.float32(1.0) / s).astype(np.float32)
    x[..., :n] = e * inv


def silu_inplace(x: np.ndarray) -> None:
    """Kernels.siluInPlaceSegment (core/Kernels.java:61-90): x / (1 + (float)exp(-x))."""
    e = np.exp(-x.astype(np.float64)).astype(np.float32)
    x[...] = x / (np.float32(1.0) + e)


def fma32(a, b, c):
    """Single-rounding fused multiply-add in float32 (a*b is exact in float64)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def rope_inplace(qk: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray, head_dim: int) -> None:
    """Kernels.ropeInPlaceSegment (core/Kernels.java:274-321), vector path.

    Per interleaved pair (a, b) at (2i, 2i+1):
        a' = fma(a, c, b * -s),  b' = fma(b, c, a * s)
    where the inner product is rounded to float before the fused add.
    """
    if qk.size % head_dim:
        raise ValueError("n is not a multiple of headDim")
    v = qk.reshape(-1, head_dim)
    a = v[:, 0::2].copy()
    b = v[:, 1::2].copy()
    c = cos_row[0::2].astype(np.float32)
    s = sin_row[0::2].astype(np.float32)
    v[:, 0::2] = fma32(a, c[None, :], (b * (-s)[None, :]).astype(np.float32))
    v[:, 1::2] = fma32(b, c[None, :], (a * s[None, :]).astype(np.float32))


def rope_tables(head_dim: int, base: float, max_ctx: int):
    """RopeCache (inference/RopeCache.java:154-177): [ctx][headDim] cos/sin, duplicated per pair.

    freq = (float) Math.pow(base, -2i/headDim) in double; angle = pos * freq
    in float; cos/sin in double then cast to float.
    """
    half = head_dim // 2
    base_f = float(np.float32(base))
    freqs = np.array([np.float32(math.pow(base_f, -2.0 * i / float(head_dim))) for i in range(half)],
                     dtype=np.float32)
    pos = np.arange(max_ctx, dtype=np.float32)[:, None]
    ang = (pos * freqs[None, :]).astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    return np.repeat(c, 2, axis=1), np.repeat(s, 2, axis=1)


# --------------------------------------------------------------------------
# Model: inference/LlamaConfig.java, KVCache.java, LlamaModel.java
# --------------------------------------------------------------------------
@dataclass
class LlamaConfig:
    """inference/LlamaConfig.java:12-53 (only the fields the decode path reads)."""
    context_length: int
    embedding_length: int
    block_count: int
    head_count: int
    head_count_kv: int
    feed_forward_length: int
    rope_freq_base: float
    rms_norm_eps: float
    vocab_size: int

    @property
    def head_dim(self) -> int:
        return self.embedding_length // self.head_count


def kv_q8_roundtrip(x: np.ndarray) -> np.ndarray:
    """The Q8_0 KV-cache rounding of the device path (no reference
    counterpart: the reference keeps K/V in FP32): per block of 32, d =
    max|x| / 127 in float32, stored as fp16 (round to nearest even); q =
    round-half-away-from-zero(x * (1 / d)) clamped to +-127 (q = 0 when d
    is 0); read back as q * fp16_to_f32_ftz(d)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.max(np.abs(x), axis=1).astype(np.float32)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    y = (x * inv[:, None]).astype(np.float32).astype(np.float64)
    q = np.clip(np.where(y >= 0, np.floor(y + 0.5), np.ceil(y - 0.5)), -127, 127).astype(np.float32)
    d16 = d.astype(np.float16).view(np.uint16)
    dd = fp16_bits_to_f32(d16).astype(np.float32)
    return (q * dd[:, None]).astype(np.float32).reshape(-1)


class KVCache:
    """inference/KVCache.java:43-95: fp32 [layer][kvHead][ctx][headDim] K and V.
    q8=True stores what the device's Q8_0 KV cache reads back."""

    def __init__(self, layers: int, kv_heads: int, head_dim: int, max_ctx: int, q8: bool = False):
        self.k = np.zeros((layers, kv_heads, max_ctx, head_dim), dtype=np.float32)
        self.v = np.zeros_like(self.k)
        self.max_ctx = max_ctx
        self.size = 0
        self.q8 = q8

    def append(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray) -> None:
        if pos >= self.max_ctx:
            raise RuntimeError(f"position {pos} exceeds maxContext {self.max_ctx}")
        hkv, hd = self.k.shape[1], self.k.shape[3]
        if self.q8:
            k, v = kv_q8_roundtrip(k), kv_q8_roundtrip(v)
        self.k[layer, :, pos, :] = np.asarray(k).reshape(hkv, hd)
        self.v[layer, :, pos, :] = np.asarray(v).reshape(hkv, hd)
        self.size = max(self.size, pos + 1)


TENSOR_DIMS = {
    # inference/Weights.java:84-112 expectedDims (logical, outer to inner)
    "token_embd.weight": lambda c: (c.vocab_size, c.embedding_length),
    "output_norm.weight": lambda c: (c.embedding_length,),
    "output.weight": lambda c: (c.vocab_size, c.embedding_length),
    "attn_q.weight": lambda c: (c.embedding_length, c.head_count * c.head_dim),
    "attn_k.weight": lambda c: (c.embedding_length, c.head_count_kv * c.head_dim),
    "attn_v.weight": lambda c: (c.embedding_length, c.head_count_kv * c.head_dim),
    "attn_output.weight": lambda c: (c.head_count * c.head_dim, c.embedding_length),
    "ffn_gate.weight": lambda c: (c.feed_forward_length, c.embedding_length),
    "ffn_up.weight": lambda c: (c.feed_forward_length, c.embedding_length),
    "ffn_down.weight": lambda c: (c.embedding_length, c.feed_forward_length),
    "attn_norm.weight": lambda c: (c.embedding_length,),
    "ffn_norm.weight": lambda c: (c.embedding_length,),
}
LAYER_TENSORS = ["attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                 "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight",
                 "attn_norm.weight", "ffn_norm.weight"]


ATTN_PROJ = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight")


def load_weight(tensors: dict, name: str, dims, layout: int = 0) -> np.ndarray:
    """Weights.wrapByName (inference/Weights.java:117-203): dequant to FP32,
    zero stand-in when the tensor is absent. With [out][in] attention bytes
    (LAYOUT_ATTN_OUT_IN) the attention matrices are transposed back to the
    reference's [in][out] reading."""
    n = int(np.prod(dims))
    if name not in tensors:
        return np.zeros(dims, dtype=np.float32)
    t = tensors[name]
    if (layout & LAYOUT_ATTN_OUT_IN) and name.endswith(ATTN_PROJ):
        return np.ascontiguousarray(dequant(t["type"], t["data"], n, layout).reshape(dims[::-1]).T)
    return dequant(t["type"], t["data"], n, layout).reshape(dims)


class LlamaModelRef:
    """LlamaModel.forwardStep restated (inference/LlamaModel.java:141-308).

    tensors: {name: {"type": ggml type code, "data": raw GGUF bytes}}.
    Attention projections keep the byte layout [in][out] (F6 in the survey):
    q[k] = sum_e B[e][k] x[e]; wo: y[e] = sum_k B[k][e] a[k].
    """

    def __init__(self, cfg: LlamaConfig, tensors: dict, layout: int = 0, kv_type: int = 0):
        self.cfg = cfg
        c = cfg
        self.tok_embd = load_weight(tensors, "token_embd.weight", TENSOR_DIMS["token_embd.weight"](c), layout)
        self.out_norm = load_weight(tensors, "output_norm.weight", TENSOR_DIMS["output_norm.weight"](c), layout)
        self.out_w = load_weight(tensors, "output.weight", TENSOR_DIMS["output.weight"](c), layout)
        self.layers = []
        for L in range(c.block_count):
            lw = {}
            for nm in LAYER_TENSORS:
                lw[nm] = load_weight(tensors, f"blk.{L}.{nm}", TENSOR_DIMS[nm](c), layout)
            self.layers.append(lw)
        self.kv = KVCache(c.block_count, c.head_count_kv, c.head_dim, c.context_length, q8=(kv_type == GGML_Q8_0))
        self.cos, self.sin = rope_tables(c.head_dim, c.rope_freq_base, c.context_length)
        self.x = np.zeros(c.embedding_length, dtype=np.float32)

    def forward_step(self, token: int, pos: int) -> np.ndarray:
        c = self.cfg
        self.x[:] = self.tok_embd[token]                      # LlamaModel.java:181-186
        for L in range(c.block_count):
            self._layer(L, pos)
        rmsnorm_inplace(self.x, self.out_norm, c.rms_norm_eps)  # :148
        return sgemv(self.out_w, self.x)                       # :155-156

    def forward_prompt(self, tokens) -> None:
        """LlamaModel.forwardPrompt (:166-175): sequential steps, returns None."""
        if len(tokens) >= self.cfg.context_length:
            raise ValueError("Prompt length exceeds contextLength")
        for i, t in enumerate(tokens):
            self.forward_step(int(t), i)

    def _layer(self, L: int, pos: int) -> None:
        c = self.cfg
        w = self.layers[L]
        hd, H, Hkv = c.head_dim, c.head_count, c.head_count_kv
        x = self.x
        rmsnorm_inplace(x, w["attn_norm.weight"], c.rms_norm_eps)        # :192 (F7: x becomes normed)
        q = (x @ w["attn_q.weight"]).astype(np.float32)                   # :196 orientation T
        k = (x @ w["attn_k.weight"]).astype(np.float32)
        v = (x @ w["attn_v.weight"]).astype(np.float32)
        rope_inplace(q, self.cos[pos], self.sin[pos], hd)                 # :209-212
        rope_inplace(k, self.cos[pos], self.sin[pos], hd)
        self.kv.append(L, pos, k, v)                                      # :216
        att = self.attention(L, pos, q)                                   # :220-221
        x += (att @ w["attn_output.weight"]).astype(np.float32)           # :224-225 orientation T
        rmsnorm_inplace(x, w["ffn_norm.weight"], c.rms_norm_eps)          # :228
        g = sgemv(w["ffn_gate.weight"], x)                                # :229
        u = sgemv(w["ffn_up.weight"], x)                                  # :230
        silu_inplace(g)                                                   # :231
        g *= u                                                            # :232
        x += sgemv(w["ffn_down.weight"], g)                               # :233-234

    def attention(self, L: int, pos: int, q: np.ndarray) -> np.ndarray:
        """LlamaModel.attention (:255-297): per q head, GQA map h*Hkv/H,
        logits = K q, times (float)(1/sqrt(hd)), softmax, out = p V."""
        c = self.cfg
        hd, H, Hkv = c.head_dim, c.head_count, c.head_count_kv
        scale = np.float32(1.0 / math.sqrt(float(hd)))
        M = pos + 1
        out = np.zeros(H * hd, dtype=np.float32)
        for h in range(H):
            kvh = h if Hkv == H else (h * Hkv) // H
            K = self.kv.k[L, kvh, :M]
            V = self.kv.v[L, kvh, :M]
            logits = (K @ q[h * hd:(h + 1) * hd]).astype(np.float32) * scale
            softmax_inplace(logits)
            out[h * hd:(h + 1) * hd] = (logits @ V).astype(np.float32)
        return out


# --------------------------------------------------------------------------
# Sampler: inference/Sampler.java:37-121 (F13)
# --------------------------------------------------------------------------
@dataclass
class SamplerConfig:
    temperature: float = 1.0
    top_k: int = 1
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    seed: int = 0


def _double_compare_key(v: float):
    """A sort key ordered as java.lang.Double.compare."""
    if math.isnan(v):
        return (2, 0.0, 0)
    return (1, v, 0 if (v == 0.0 and math.copysign(1.0, v) < 0) else 1)


def sample(logits: np.ndarray, history, cfg: SamplerConfig) -> int:
    """Sampler.sample: penalty, greedy fast path, stable descending sort,
    top-k, top-p on running/total >= topP, renormalise, CDF scan with
    r = new Random(seed).nextFloat()."""
    logits = np.asarray(logits, dtype=np.float32)
    vocab = logits.size
    f32 = np.float32
    if cfg.repetition_penalty != 1.0 and history is not None and len(history) > 0:
        p = f32(cfg.repetition_penalty)
        for tok in history:
            if 0 <= tok < vocab:
                if logits[tok] > 0:
                    logits[tok] = f32(logits[tok] / p)
                else:
                    logits[tok] = f32(logits[tok] * p)
    if cfg.temperature == 0.0 or (cfg.top_k == 1 and cfg.top_p >= 1.0):
        best, best_score = 0, logits[0]
        for i in range(1, vocab):
            if logits[i] > best_score:
                best_score, best = logits[i], i
        return best
    inv_t = f32(f32(1.0) / f32(cfg.temperature))
    adj = (logits * inv_t).astype(np.float32)
    # Comparator.comparingDouble(..).reversed() under List.sort: stable,
    # descending in Double.compare's order (NaN above +inf, -0.0 below 0.0);
    # equal values keep ascending index order
    order = sorted(range(vocab), key=lambda i: _double_compare_key(float(adj[i])), reverse=True)
    top_k = min(cfg.top_k, vocab)
    max_logit = adj[order[0]]
    probs = np.zeros(top_k, dtype=np.float32)
    sum_exp = f32(0.0)
    for i in range(top_k):
        pr = f32(math.exp(float(f32(adj[order[i]] - max_logit))))
        probs[i] = pr
        sum_exp = f32(sum_exp + pr)
    cutoff = top_k
    if cfg.top_p < 1.0:
        running = f32(0.0)
        total = sum_exp
        for i in range(top_k):
            running = f32(running + probs[i])
            if f32(running / total) >= f32(cfg.top_p):
                cutoff = i + 1
                break
    new_sum = f32(0.0)
    for i in range(cutoff):
        new_sum = f32(new_sum + probs[i])
    for i in range(cutoff):
        probs[i] = f32(probs[i] / new_sum)
    if cfg.seed == 0:
        raise ValueError("seed 0 selects a non-deterministic RNG in the reference; pass a seed")
    r = f32(JavaRandom(cfg.seed).next_float())
    cum = f32(0.0)
    for i in range(cutoff):
        cum = f32(cum + probs[i])
        if r <= cum:
            return order[i]
    return order[cutoff - 1]
