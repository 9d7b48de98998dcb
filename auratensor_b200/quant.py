"""Device mirror of the reference's block codecs (quant/Q4_0.java,
quant/Q8_0.java, quant/QuantBlock.java) and the device-resident quantized
matrix used by the fused GEMV.

Block tensors are raw GGUF bytes in a uint8 CUDA tensor. ``dot`` follows
``dequantToFloat`` semantics over all 32 elements of each block (the
reference's SIMD ``dot`` covers only part of each block below 512-bit
vectors, quant/Q4_0.java:71-87).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import GGML_Q4_0, GGML_Q6_K, GGML_Q8_0, ORIENT_N, ORIENT_T, IllegalArgumentException, call
from .core import context, ptr

BLOCK_SIZE = 32


class QuantBlock:
    """quant/QuantBlock.java:27-39."""
    BLOCK_SIZE = 32

    @staticmethod
    def bytesPerBlock(ggml_type: int) -> int:
        if ggml_type == GGML_Q8_0:
            return 34
        if ggml_type == GGML_Q4_0:
            return 18
        if ggml_type == GGML_Q6_K:
            return 210
        raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, f"Not a block-quantized type: {ggml_type}")

    @staticmethod
    def elementsPerBlock(ggml_type: int) -> int:
        return 256 if ggml_type == GGML_Q6_K else 32


def _check(src: torch.Tensor, n: int, bpb: int):
    if not src.is_cuda or src.dtype != torch.uint8:
        raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "blocks must be a uint8 CUDA tensor")
    if src.numel() < (n // BLOCK_SIZE) * bpb:
        raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "block buffer too small")


class _Codec:
    TYPE = -1
    BPB = 0
    _DEQ = ""
    _DOT = ""

    @classmethod
    def dequantToFloat(cls, src: torch.Tensor, dst: torch.Tensor | None, numElements: int) -> torch.Tensor:
        _check(src, numElements, cls.BPB)
        if dst is None:
            dst = torch.empty(numElements, dtype=torch.float32, device=src.device)
        call(cls._DEQ, context(src.device.index), ptr(src), ptr(dst), int(numElements))
        return dst

    @classmethod
    def dot(cls, q: torch.Tensor, x: torch.Tensor, numElements: int) -> float:
        _check(q, numElements, cls.BPB)
        out = torch.empty(1, dtype=torch.float32, device=q.device)
        call(cls._DOT, context(q.device.index), ptr(q), ptr(x.contiguous()), int(numElements), ptr(out))
        return float(out.item())


class Q4_0(_Codec):
    """quant/Q4_0.java: 18-byte blocks, w = (q - 8) * d, interleaved nibbles."""
    TYPE, BPB, _DEQ, _DOT = GGML_Q4_0, 18, "at_q4_0_dequant", "at_q4_0_dot"


class Q8_0(_Codec):
    """quant/Q8_0.java: 34-byte blocks, w = q * d."""
    TYPE, BPB, _DEQ, _DOT = GGML_Q8_0, 34, "at_q8_0_dequant", "at_q8_0_dot"


class Q6_K:
    """quant/Q6_K.java: 210-byte blocks of 256 elements, (d * scale) * (q - 32)."""
    TYPE, BPB = GGML_Q6_K, 210

    @classmethod
    def dequantToFloat(cls, src: torch.Tensor, dst: torch.Tensor | None, numElements: int) -> torch.Tensor:
        if not src.is_cuda or src.dtype != torch.uint8:
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "blocks must be a uint8 CUDA tensor")
        if numElements % 256 or src.numel() < (numElements // 256) * cls.BPB:
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "bad Q6_K element count or buffer size")
        if dst is None:
            dst = torch.empty(numElements, dtype=torch.float32, device=src.device)
        call("at_q6_k_dequant", context(src.device.index), ptr(src), ptr(dst), int(numElements))
        return dst


class QMatrix:
    """Raw GGUF block matrix re-laid-out on the device for the fused GEMV.

    orient N: y[b][r] = sum_c W[r][c] x[b][c] (weights stored [out][in]);
    orient T: y[b][c] = sum_r W[r][c] x[b][r] (weights stored [in][out]).
    """

    def __init__(self, ggml_type: int, orient: int, rows: int, cols: int, blocks, layout: int = 0):
        """layout: _lib.LAYOUT_Q4_SPLIT_HALVES reads Q4_0 blocks in llama.cpp's
        nibble order (stored and exported in the reference's order)."""
        self.type, self.orient, self.rows, self.cols = ggml_type, orient, int(rows), int(cols)
        self._h = C.c_void_p()
        if isinstance(blocks, torch.Tensor):
            if blocks.is_cuda:
                dev = blocks.device.index
                src, on_dev = ptr(blocks.contiguous()), 1
                keep = blocks
            else:
                dev = torch.cuda.current_device()
                keep = blocks.contiguous()
                src, on_dev = C.c_void_p(keep.data_ptr()), 0
        else:
            import numpy as np
            keep = np.ascontiguousarray(blocks)
            dev = torch.cuda.current_device()
            src, on_dev = C.c_void_p(keep.ctypes.data), 0
        self.device = dev
        call("at_qmat_create_ex", context(dev), ggml_type, orient, int(layout), self.rows, self.cols, src, on_dev,
             C.byref(self._h))
        del keep

    @property
    def out_features(self) -> int:
        return self.rows if self.orient == ORIENT_N else self.cols

    @property
    def in_features(self) -> int:
        return self.cols if self.orient == ORIENT_N else self.rows

    def gemv(self, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        """x: [batch][in] float32 CUDA tensor (batch 1..8) -> y: [batch][out]."""
        x2 = x.reshape(-1, self.in_features).contiguous()
        b = x2.shape[0]
        if y is None:
            y = torch.empty((b, self.out_features), dtype=torch.float32, device=x.device)
        call("at_gemv", context(self.device), self._h, ptr(x2), ptr(y), b)
        return y

    def gemm(self, x: torch.Tensor, y: torch.Tensor | None = None) -> torch.Tensor:
        """Prompt-chunk GEMM on the tensor cores: x [tokens][in] float32 CUDA
        tensor -> y [tokens][out], bf16 operands with FP32 sums."""
        x2 = x.reshape(-1, self.in_features).contiguous()
        t = x2.shape[0]
        if y is None:
            y = torch.empty((t, self.out_features), dtype=torch.float32, device=x.device)
        call("at_gemm_tc", context(self.device), self._h, ptr(x2), ptr(y), t)
        return y

    def export_blocks(self) -> torch.Tensor:
        bpb = QuantBlock.bytesPerBlock(self.type)
        per = QuantBlock.elementsPerBlock(self.type)
        out = torch.empty(self.rows * (self.cols // per) * bpb, dtype=torch.uint8, device=f"cuda:{self.device}")
        call("at_qmat_export", context(self.device), self._h, ptr(out))
        return out

    def close(self):
        if self._h:
            call("at_qmat_destroy", self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["QuantBlock", "Q4_0", "Q8_0", "Q6_K", "QMatrix", "ORIENT_N", "ORIENT_T"]
