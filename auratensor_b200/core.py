"""Device-backed mirror of the reference's core package (core/Tensor.java,
core/Kernels.java, core/Fp16.java, core/DType.java).

``Tensor`` keeps its elements in HBM (a CUDA tensor owned through PyTorch's
allocator); ``Kernels`` runs each op through the C ABI of
libauratensor_cuda.so on the caller's current CUDA stream. Argument checks and
exception classes follow the reference so code written against it reads the
same. Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes as C
import enum
import threading

import torch

from . import _lib
from ._lib import IllegalArgumentException, call


class DType(enum.Enum):
    """core/DType.java:11-25."""
    FP32 = 4
    FP16 = 2
    INT8 = 1
    INT4 = 1

    def bytes_per_element(self) -> int:
        return self.value


_TORCH = {DType.FP32: torch.float32, DType.FP16: torch.float16, DType.INT8: torch.int8}

_ctx_lock = threading.Lock()
_ctxs: dict = {}


def context(device: int | None = None) -> int:
    """The per-device at_ctx of this process, bound to torch's current stream."""
    if device is None:
        device = torch.cuda.current_device()
    with _ctx_lock:
        ctx = _ctxs.get(device)
        if ctx is None:
            p = C.c_void_p()
            call("at_ctx_create", device, C.byref(p))
            ctx = _ctxs[device] = p.value
    call("at_ctx_set_stream", ctx, C.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    return ctx


def ptr(t: torch.Tensor) -> C.c_void_p:
    if not t.is_cuda:
        raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "tensor is not on a CUDA device")
    return C.c_void_p(t.data_ptr())


class Tensor:
    """core/Tensor.java: rank 1-3 row-major tensor; here its memory is HBM."""

    def __init__(self, data: torch.Tensor, dtype: DType, shape):
        shape = tuple(int(s) for s in shape)
        if not 1 <= len(shape) <= 3:
            raise IllegalArgumentException(
                _lib.AT_ERR_INVALID_ARG, f"AuraTensor supports rank 1, 2, or 3 tensors (got rank {len(shape)})")
        for s in shape:
            if s <= 0:
                raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, f"All dimensions must be positive, got {s}")
        self._data = data
        self._dtype = dtype
        self._shape = shape

    # Tensor.allocate* (core/Tensor.java:73-94)
    @classmethod
    def allocate(cls, dtype: DType, *shape) -> "Tensor":
        n = 1
        for s in shape:
            n *= int(s)
        if n <= 0:
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "All dimensions must be positive")
        data = torch.zeros(n, dtype=_TORCH.get(dtype, torch.uint8), device="cuda")
        return cls(data, dtype, shape)

    @classmethod
    def allocate1D(cls, dtype, n):
        return cls.allocate(dtype, n)

    @classmethod
    def allocate2D(cls, dtype, rows, cols):
        return cls.allocate(dtype, rows, cols)

    @classmethod
    def allocate3D(cls, dtype, d0, d1, d2):
        return cls.allocate(dtype, d0, d1, d2)

    # Tensor.wrap (core/Tensor.java:104-111): wraps existing device memory.
    @classmethod
    def wrap(cls, data: torch.Tensor, dtype: DType, shape) -> "Tensor":
        n = 1
        for s in shape:
            n *= int(s)
        if data.numel() * data.element_size() < n * dtype.bytes_per_element():
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "segment too small for shape")
        return cls(data.reshape(-1), dtype, shape)

    def data(self) -> torch.Tensor:
        return self._data

    def dtype(self) -> DType:
        return self._dtype

    def shape(self):
        return list(self._shape)

    def rank(self) -> int:
        return len(self._shape)

    def numElements(self) -> int:
        n = 1
        for s in self._shape:
            n *= s
        return n

    def _offset(self, idx) -> int:
        if len(idx) != len(self._shape):
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "index rank mismatch")
        off = 0
        for i, s in zip(idx, self._shape):
            if not 0 <= i < s:
                raise IndexError(f"index {i} out of bounds for dim {s}")
            off = off * s + i
        return off

    def getFloat(self, *idx) -> float:
        return float(self._data[self._offset(idx)].item())

    def setFloat(self, v: float, *idx) -> None:
        self._data[self._offset(idx)] = v

    def close(self) -> None:
        self._data = None


class Fp16:
    """core/Fp16.java:19-37 on the device (subnormals flush to zero)."""

    @staticmethod
    def toFloat(bits: torch.Tensor) -> torch.Tensor:
        src = bits.contiguous().view(torch.int16)
        out = torch.empty(src.numel(), dtype=torch.float32, device=src.device)
        call("at_fp16_to_f32", context(src.device.index), ptr(src), ptr(out), src.numel())
        return out


def _fp32(t: Tensor, name: str):
    if t.dtype() != DType.FP32:
        raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, f"{name} requires FP32 tensor")


class Kernels:
    """core/Kernels.java ops, launched on the GPU."""

    @staticmethod
    def siluInPlace(x: Tensor) -> None:
        _fp32(x, "siluInPlace")
        Kernels.siluInPlaceSegment(x.data(), x.numElements())

    @staticmethod
    def siluInPlaceSegment(seg: torch.Tensor, n: int) -> None:
        call("at_silu", context(), ptr(seg), int(n))

    @staticmethod
    def rmsNormInPlace(x: Tensor, weight: Tensor, eps: float) -> None:
        if x.dtype() != DType.FP32 or weight.dtype() != DType.FP32:
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "rmsNorm requires FP32 tensors")
        if x.rank() not in (1, 2):
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "rmsNorm requires rank 1 or 2 tensors")
        d = x.shape()[-1]
        if weight.numElements() != d:
            raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG,
                                           f"weight length {weight.numElements()} != last dim {d}")
        call("at_rmsnorm", context(), ptr(x.data()), ptr(weight.data()), float(eps), x.numElements() // d, d)

    @staticmethod
    def softmaxInPlace(x: Tensor) -> None:
        _fp32(x, "softmax")
        d = x.shape()[-1]
        call("at_softmax", context(), ptr(x.data()), x.numElements() // d, d)

    @staticmethod
    def softmaxInPlaceSegment(seg: torch.Tensor, n: int) -> None:
        call("at_softmax", context(), ptr(seg), 1, int(n))

    @staticmethod
    def ropeInPlace(qk: Tensor, cos: Tensor, sin: Tensor, head_dim: int) -> None:
        _fp32(qk, "ropeInPlace")
        Kernels.ropeInPlaceSegment(qk.data(), cos.data(), sin.data(), head_dim, qk.numElements())

    @staticmethod
    def ropeInPlaceSegment(qk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, head_dim: int, n: int) -> None:
        call("at_rope", context(), ptr(qk), ptr(cos), ptr(sin), int(head_dim), int(n))

    @staticmethod
    def sgemv(A, x, y, M: int | None = None, K: int | None = None) -> None:
        """Kernels.sgemv(Tensor A, Tensor x, Tensor y) or the segment form (a, x, y, M, K)."""
        if isinstance(A, Tensor):
            if A.rank() != 2 or x.rank() != 1 or y.rank() != 1:
                raise IllegalArgumentException(
                    _lib.AT_ERR_INVALID_ARG, f"sgemv: rank mismatch A={A.rank()} x={x.rank()} y={y.rank()}")
            M, K = A.shape()
            if x.numElements() != K or y.numElements() != M:
                raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "sgemv: dim mismatch")
            A, x, y = A.data(), x.data(), y.data()
        call("at_sgemv", context(), ptr(A), ptr(x), ptr(y), int(M), int(K))

    @staticmethod
    def sgemm(A, B, Cm, M: int | None = None, K: int | None = None, N: int | None = None) -> None:
        if isinstance(A, Tensor):
            if A.rank() != 2 or B.rank() != 2 or Cm.rank() != 2:
                raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "sgemm: rank mismatch")
            M, K = A.shape()
            N = B.shape()[1]
            if B.shape()[0] != K or Cm.shape()[0] != M or Cm.shape()[1] != N:
                raise IllegalArgumentException(_lib.AT_ERR_INVALID_ARG, "sgemm: dim mismatch")
            A, B, Cm = A.data(), B.data(), Cm.data()
        call("at_sgemm", context(), ptr(A), ptr(B), ptr(Cm), int(M), int(K), int(N))
