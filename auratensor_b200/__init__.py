"""AuraTensor-B200: the quantized-matvec decode path of AuraTensor on B200 (sm_100a).

Modules mirror the reference's packages: ``core`` (Tensor, Kernels, Fp16),
``quant`` (Q4_0, Q8_0, QuantBlock, QMatrix), ``gguf`` (GgufFile reader and
writer), ``inference`` (LlamaConfig, LlamaModel, KVCache, Sampler) and ``tp``
(tensor-parallel bootstrap). All compute runs in libauratensor_cuda.so.
"""
from ._lib import LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
