"""Device mirror of the reference's inference package: LlamaConfig, Weights
loading, LlamaModel, KVCache and Sampler (inference/*.java).

``LlamaModel`` owns an ``at_model`` of libauratensor_cuda.so: the raw Q4_0 /
Q8_0 blocks are uploaded once and every forward step runs as one CUDA graph.
``forwardStep`` returns the logits as a float32 numpy array, as the reference
returns ``float[]``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import ModelConfig, call
from .core import context
from .gguf import GgufFile


@dataclass
class LlamaConfig:
    """inference/LlamaConfig.java:12-53."""
    architecture: str = "llama"
    contextLength: int = 4096
    embeddingLength: int = 4096
    blockCount: int = 32
    headCount: int = 32
    headCountKv: int = 32
    feedForwardLength: int = 11008
    ropeFrequencyBase: float = 10000.0
    rmsNormEpsilon: float = 1e-5
    vocabSize: int = 32000

    def headDim(self) -> int:
        if self.headCount == 0:
            raise _lib.IllegalStateException(_lib.AT_ERR_STATE, "headCount == 0")
        return self.embeddingLength // self.headCount

    @classmethod
    def fromGguf(cls, m) -> "LlamaConfig":
        arch = m.string_or_default("general.architecture", "llama")
        n_emb = m.long_or_default(arch + ".embedding_length", 4096)
        n_heads = m.long_or_default(arch + ".attention.head_count", 32)
        rope_default = 500000.0 if ("llama" in arch and n_emb >= 4096) else 10000.0
        return cls(
            architecture=arch,
            contextLength=m.long_or_default(arch + ".context_length", 4096),
            embeddingLength=n_emb,
            blockCount=m.long_or_default(arch + ".block_count", 32),
            headCount=n_heads,
            headCountKv=m.long_or_default(arch + ".attention.head_count_kv", n_heads),
            feedForwardLength=m.long_or_default(arch + ".feed_forward_length", 11008),
            ropeFrequencyBase=float(np.float32(m.float_or_default(arch + ".rope.freq_base", rope_default))),
            rmsNormEpsilon=float(np.float32(m.float_or_default(arch + ".attention.layer_norm_rms_epsilon", 1e-5))),
            vocabSize=m.long_or_default(arch + ".vocab_size", m.long_or_default("tokenizer.ggml.vocab_size", 32000)),
        )

    @classmethod
    def fromShape(cls, s) -> "LlamaConfig":
        return cls("llama", s.ctx, s.dim, s.n_layers, s.n_heads, s.n_kv_heads, s.ffn, float(s.rope_theta),
                   float(s.eps), s.vocab)

    def to_c(self, max_batch: int = 1, layout: int = 0, kv_type: int = 0) -> ModelConfig:
        return ModelConfig(self.contextLength, self.embeddingLength, self.blockCount, self.headCount,
                           self.headCountKv, self.feedForwardLength, self.vocabSize, self.ropeFrequencyBase,
                           self.rmsNormEpsilon, max_batch, layout, kv_type, 0)


class KVCache:
    """View of the device KV cache of one sequence slot (inference/KVCache.java:29-111)."""

    def __init__(self, model: "LlamaModel", slot: int = 0):
        self._m, self._slot = model, slot
        c = model.config
        self._dims = (c.blockCount, c.headCountKv // model.world, c.headDim(), c.contextLength)

    def size(self) -> int:
        v = C.c_int64()
        call("at_model_kv_size", self._m._h, self._slot, C.byref(v))
        return v.value

    def maxContext(self) -> int:
        return self._dims[3]

    def blockCount(self) -> int:
        return self._dims[0]

    def headCountKv(self) -> int:
        return self._dims[1]

    def headDim(self) -> int:
        return self._dims[2]

    def rowBytes(self) -> int:
        return self._dims[3] * self._dims[2] * 4

    def offsetOf(self, layer, kv_head, position, dim) -> int:
        """KVCache.offsetOf through at_model_kv_offset (same checks and messages)."""
        v = C.c_int64()
        call("at_model_kv_offset", self._m._h, int(layer), int(kv_head), int(position), int(dim), C.byref(v))
        return v.value

    def append(self, layer: int, position: int, kSlice, vSlice) -> None:
        """KVCache.append: headCountKv x headDim floats of K and of V at `position`."""
        k = np.ascontiguousarray(np.asarray(kSlice, dtype=np.float32).reshape(-1))
        v = np.ascontiguousarray(np.asarray(vSlice, dtype=np.float32).reshape(-1))
        n = self._dims[1] * self._dims[2]
        if k.size != n or v.size != n:
            raise _lib.IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, f"K/V slices must hold {n} floats")
        call("at_model_kv_append", self._m._h, self._slot, int(layer), int(position), k.ctypes.data_as(C.c_void_p),
             v.ctypes.data_as(C.c_void_p))

    def read(self, layer: int, kv_head: int, position: int):
        hd = self._dims[2]
        k = np.empty(hd, dtype=np.float32)
        v = np.empty(hd, dtype=np.float32)
        call("at_model_kv_read", self._m._h, self._slot, layer, kv_head, position,
             k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p))
        return k, v

    def reset(self) -> None:
        call("at_model_kv_reset", self._m._h, self._slot)


class LlamaModel:
    """inference/LlamaModel.java:41-381 on the device.

    Build from a GGUF path (``LlamaModel.fromGguf``), or from a config plus a
    {name: raw bytes} tensor table (``LlamaModel(config, tensors)``); tensors
    may be numpy arrays / bytes (uploaded once) or uint8 CUDA tensors.
    Under tensor parallelism pass ``ctx`` from ``tp.init_tp_context``.
    """

    def __init__(self, config: LlamaConfig, tensors: dict | None = None, max_batch: int = 1, ctx=None,
                 world: int = 1, layout: int = 0, kv_type: int = 0):
        """layout: byte layout of the tensors (_lib.LAYOUT_*; 0 is the
        reference's, _lib.LAYOUT_LLAMA_CPP reads llama.cpp exports).
        kv_type: KV cache storage, 0 (F32, the reference's) or 8 (Q8_0)."""
        self.config = config
        self.max_batch = max_batch
        self.world = world
        self._ctx = ctx if ctx is not None else context()
        self._h = C.c_void_p()
        cfg = config.to_c(max_batch, layout, kv_type)
        call("at_model_create", self._ctx, C.byref(cfg), C.byref(self._h))
        self._logits = _host_logits(max_batch, config.vocabSize)
        if tensors is not None:
            for name, t in tensors.items():
                self.setTensor(name, t["type"], t["data"])
            self.finalize()

    @classmethod
    def fromGguf(cls, path: str, max_batch: int = 1, layout: int = 0, kv_type: int = 0) -> "LlamaModel":
        with GgufFile.open(path) as g:
            cfg = LlamaConfig.fromGguf(g.metadata)
        self = cls.__new__(cls)
        self.config = cfg
        self.max_batch = max_batch
        self.world = 1
        self._ctx = context()
        self._h = C.c_void_p()
        call("at_model_load_gguf_ex", self._ctx, path.encode(), max_batch, int(layout), int(kv_type), C.byref(self._h))
        self._logits = _host_logits(max_batch, cfg.vocabSize)
        return self

    def setTensor(self, name: str, ggml_type: int, data) -> None:
        if isinstance(data, torch.Tensor) and data.is_cuda:
            d = data.contiguous()
            call("at_model_set_tensor", self._h, name.encode(), ggml_type, C.c_void_p(d.data_ptr()),
                 d.numel() * d.element_size(), 1)
        else:
            arr = np.ascontiguousarray(np.frombuffer(memoryview(data), dtype=np.uint8))
            call("at_model_set_tensor", self._h, name.encode(), ggml_type, arr.ctypes.data_as(C.c_void_p),
                 arr.nbytes, 0)

    def finalize(self) -> None:
        call("at_model_finalize", self._h)

    def kvCache(self, slot: int = 0) -> KVCache:
        return KVCache(self, slot)

    def forwardStep(self, tokenId: int, position: int) -> np.ndarray:
        """LlamaModel.forwardStep: logits over the vocabulary (host array)."""
        out = self._logits[0]
        call("at_model_forward_step", self._h, int(tokenId), int(position), out.ctypes.data_as(C.c_void_p))
        return out

    def forwardStepDevice(self, tokenId: int, position: int) -> None:
        """forwardStep without copying the logits to the host."""
        call("at_model_forward_step", self._h, int(tokenId), int(position), None)

    def forwardPrompt(self, promptTokenIds) -> None:
        arr = np.ascontiguousarray(np.asarray(promptTokenIds, dtype=np.int32))
        call("at_model_forward_prompt", self._h, arr.ctypes.data_as(C.c_void_p), int(arr.size))
        return None

    def forwardBatch(self, tokens, positions, copy_logits: bool = True) -> np.ndarray | None:
        """One decode step of len(tokens) independent sequences (slot b <- tokens[b])."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int64))
        b = int(t.size)
        out = self._logits[:b] if copy_logits else None
        call("at_model_forward_batch", self._h, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p), b,
             out.ctypes.data_as(C.c_void_p) if out is not None else None)
        return out

    def logitsDevice(self) -> torch.Tensor:
        """The last step's logits [max_batch][vocab] as a CUDA tensor view."""
        p = C.c_void_p()
        call("at_model_logits_device", self._h, C.byref(p))
        n = self.max_batch * self.config.vocabSize
        return _device_view(p.value, n, torch.cuda.current_device()).view(self.max_batch, self.config.vocabSize)

    def generate(self, firstToken: int, startPos: int, nSteps: int, wait: bool = True) -> np.ndarray | None:
        """Greedy decode of slot 0 on the device: nSteps tokens, no host round trip per step."""
        if not wait:
            call("at_model_generate", self._h, int(firstToken), int(startPos), int(nSteps), None)
            return None
        out = np.empty(max(1, nSteps), dtype=np.int32)
        call("at_model_generate", self._h, int(firstToken), int(startPos), int(nSteps),
             out.ctypes.data_as(C.c_void_p))
        return out[:nSteps]

    def forwardPromptSlot(self, slot: int, promptTokenIds) -> None:
        """forwardPrompt into KV slot `slot` (the batched prompt path)."""
        arr = np.ascontiguousarray(np.asarray(promptTokenIds, dtype=np.int32))
        call("at_model_forward_prompt_slot", self._h, int(slot), arr.ctypes.data_as(C.c_void_p), int(arr.size))

    def sample(self, configs, histories=None) -> np.ndarray:
        """Sampler.sample on the device for rows 0..len(configs)-1 of the last
        step's logits (row b with configs[b] and penalty history histories[b]);
        the penalty is applied to the device logits in place."""
        cfgs, keep = _sampler_array(configs, histories)
        out = np.empty(len(configs), dtype=np.int32)
        call("at_model_sample", self._h, len(configs), C.cast(cfgs, C.c_void_p), out.ctypes.data_as(C.c_void_p))
        del keep
        return out

    def generateSampled(self, firstTokens, startPositions, nSteps: int, configs, histories=None) -> np.ndarray:
        """Batched sampled decode on the device: [batch][nSteps] tokens, row b in
        KV slot b with configs[b]; each row's history grows by its samples."""
        t = np.ascontiguousarray(np.asarray(firstTokens, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(startPositions, dtype=np.int64))
        b = int(t.size)
        cfgs, keep = _sampler_array(configs, histories)
        out = np.empty((b, max(1, nSteps)), dtype=np.int32)
        call("at_model_generate_sampled", self._h, b, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
             int(nSteps), C.cast(cfgs, C.c_void_p), out.ctypes.data_as(C.c_void_p))
        del keep
        return out[:, :nSteps]

    def profileStep(self, tokenId: int, position: int) -> dict:
        """Per-kernel-class device time (ms) and launch counts of one eager step."""
        ms = np.zeros(len(_lib.PROF_CLASSES), dtype=np.float32)
        n = np.zeros(len(_lib.PROF_CLASSES), dtype=np.int32)
        call("at_model_profile_step", self._h, int(tokenId), int(position), ms.ctypes.data_as(C.c_void_p),
             n.ctypes.data_as(C.c_void_p))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(_lib.PROF_CLASSES)}

    def profileBatch(self, tokens, positions) -> dict:
        """profileStep for one batched step of slots 0..len(tokens)-1."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int64))
        ms = np.zeros(len(_lib.PROF_CLASSES), dtype=np.float32)
        n = np.zeros(len(_lib.PROF_CLASSES), dtype=np.int32)
        call("at_model_profile_batch", self._h, int(t.size), t.ctypes.data_as(C.c_void_p),
             p.ctypes.data_as(C.c_void_p), ms.ctypes.data_as(C.c_void_p), n.ctypes.data_as(C.c_void_p))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(_lib.PROF_CLASSES)}

    def stream(self) -> int:
        p = C.c_void_p()
        call("at_ctx_stream", self._ctx, C.byref(p))
        return p.value or 0

    def persistentStep(self) -> bool:
        """True when batch-1 steps run as the one-launch persistent kernel."""
        v = C.c_int()
        call("at_model_step_kernel", self._h, C.byref(v))
        return bool(v.value)

    def stepStamps(self, tokenId: int, position: int) -> np.ndarray:
        """One persistent-kernel step with per-job %globaltimer stamps:
        [n_ctas][5 * layers + 1][4] nanoseconds (job start, activations staged,
        units done, job end)."""
        jobs = 5 * self.config.blockCount + 1
        n = 1024 * jobs * 4
        buf = np.zeros(n, dtype=np.uint64)
        nc = C.c_int()
        call("at_model_step_stamps", self._h, int(tokenId), int(position), buf.ctypes.data_as(C.c_void_p), n,
             C.byref(nc))
        return buf[: nc.value * jobs * 4].reshape(nc.value, jobs, 4)

    def argmax(self, batch: int = 1) -> np.ndarray:
        out = np.empty(batch, dtype=np.int32)
        call("at_model_argmax", self._h, batch, out.ctypes.data_as(C.c_void_p))
        return out

    def close(self) -> None:
        if self._h:
            call("at_model_destroy", self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _host_logits(rows: int, vocab: int) -> np.ndarray:
    """Page-locked host buffer for the logits copies (plain memory without a GPU)."""
    if torch.cuda.is_available():
        return torch.empty((rows, vocab), dtype=torch.float32, pin_memory=True).numpy()
    return np.empty((rows, vocab), dtype=np.float32)


def _device_view(addr: int, n: int, device: int) -> torch.Tensor:
    """A float32 CUDA tensor aliasing n floats at a device address owned by the library."""

    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (addr, False), "version": 3}

    return torch.as_tensor(_Holder(), device=f"cuda:{device}")


@dataclass
class SamplerConfig:
    """Sampler.Config (inference/Sampler.java:20-30)."""
    temperature: float = 1.0
    topK: int = 1
    topP: float = 1.0
    repetitionPenalty: float = 1.0
    seed: int = 0

    @staticmethod
    def greedy() -> "SamplerConfig":
        return SamplerConfig(1.0, 1, 1.0, 1.0, 0)


def _sampler_array(configs, histories):
    """An at_sampler_config array; the history arrays it points to are returned to be kept alive."""
    n = len(configs)
    arr = (_lib.SamplerConfigC * n)()
    keep = []
    for b, c in enumerate(configs):
        h = None if histories is None or histories[b] is None else np.ascontiguousarray(
            np.asarray(histories[b], dtype=np.int32))
        keep.append(h)
        arr[b] = _lib.SamplerConfigC(float(c.temperature), int(c.topK), float(c.topP), float(c.repetitionPenalty),
                                     int(c.seed), h.ctypes.data if h is not None and h.size else None,
                                     0 if h is None else int(h.size), 0)
    return arr, (arr, keep)


class Sampler:
    """Sampler.sample (inference/Sampler.java:37-121), native host code."""
    Config = SamplerConfig

    @staticmethod
    def sample(logits, history, config: SamplerConfig) -> int:
        arr = np.asarray(logits, dtype=np.float32)
        if not arr.flags.writeable or not arr.flags.c_contiguous:
            arr = np.ascontiguousarray(arr).copy()
        h = None if history is None else np.ascontiguousarray(np.asarray(history, dtype=np.int32))
        out = C.c_int()
        call("at_sample", arr.ctypes.data_as(C.c_void_p), int(arr.size),
             h.ctypes.data_as(C.c_void_p) if h is not None else None, 0 if h is None else int(h.size),
             float(config.temperature), int(config.topK), float(config.topP), float(config.repetitionPenalty),
             int(config.seed), C.byref(out))
        if isinstance(logits, np.ndarray) and arr is not logits and logits.flags.writeable:
            logits[...] = arr  # the reference mutates logits in place (repetition penalty)
        return out.value
