"""ctypes binding of libauratensor_cuda.so (the C ABI declared in include/auratensor.h).

The library is loaded from the package's in-tree ``lib/`` directory. There is
no fallback: if it is missing, or a call is made without a CUDA device, the
call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libauratensor_cuda.so")

AT_OK = 0
AT_ERR_INVALID_ARG = -1
AT_ERR_STATE = -2
AT_ERR_UNSUPPORTED = -3
AT_ERR_IO = -4
AT_ERR_CUDA = -5
AT_ERR_NCCL = -6
AT_ERR_OOM = -7
AT_ERR_TIMEOUT = -8

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q6_K = 0, 1, 2, 8, 14
# byte layouts of a model's tensors (include/auratensor.h AT_LAYOUT_*)
LAYOUT_REFERENCE, LAYOUT_Q4_SPLIT_HALVES, LAYOUT_ATTN_OUT_IN, LAYOUT_LLAMA_CPP = 0, 1, 2, 3
ORIENT_N, ORIENT_T = 0, 1
PROF_CLASSES = ["embed", "qkv", "attn", "wo", "ffn_up", "ffn_down", "lm_head", "argmax", "comm"]


class AtError(RuntimeError):
    """Base class; subclasses mirror the reference's exception classes."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class IllegalArgumentException(AtError, ValueError):
    pass


class IllegalStateException(AtError):
    pass


class UnsupportedOperationException(AtError, NotImplementedError):
    pass


class GgufIOException(AtError, IOError):
    pass


_EXC = {AT_ERR_INVALID_ARG: IllegalArgumentException, AT_ERR_STATE: IllegalStateException,
        AT_ERR_UNSUPPORTED: UnsupportedOperationException, AT_ERR_IO: GgufIOException}


class ModelConfig(C.Structure):
    _fields_ = [("context_length", C.c_int64), ("embedding_length", C.c_int64), ("block_count", C.c_int64),
                ("head_count", C.c_int64), ("head_count_kv", C.c_int64), ("feed_forward_length", C.c_int64),
                ("vocab_size", C.c_int64), ("rope_freq_base", C.c_float), ("rms_norm_eps", C.c_float),
                ("max_batch", C.c_int32), ("layout", C.c_int32), ("kv_type", C.c_int32), ("reserved", C.c_int32)]


class ShardRegion(C.Structure):
    """at_shard_region: the part of a weight tensor one tensor-parallel rank keeps."""
    _fields_ = [("target", C.c_int32), ("orient", C.c_int32), ("rows", C.c_int64), ("cols", C.c_int64),
                ("local_rows", C.c_int64), ("local_cols", C.c_int64), ("src_row0", C.c_int64),
                ("src_col0", C.c_int64), ("n_rows", C.c_int64), ("n_cols", C.c_int64), ("dst_row0", C.c_int64),
                ("dst_col0", C.c_int64)]


SHARD_NONE, SHARD_TOKEN_EMBD, SHARD_OUTPUT, SHARD_QKV, SHARD_WO, SHARD_W1, SHARD_W3, SHARD_W2, SHARD_NORM = range(-1, 8)


class SamplerConfigC(C.Structure):
    """at_sampler_config: Sampler.Config plus a host penalty history."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("seed", C.c_int64), ("history", C.c_void_p),
                ("history_len", C.c_int32), ("reserved", C.c_int32)]


_vp, _i, _i64, _sz, _f = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
_PP = C.POINTER(C.c_void_p)

# name -> argtypes (every entry point declared in include/auratensor.h)
SIGNATURES = {
    "at_last_error": [C.c_char_p, _sz],
    "at_device_count": [C.POINTER(C.c_int)],
    "at_ctx_create": [_i, _PP],
    "at_ctx_destroy": [_vp],
    "at_ctx_synchronize": [_vp],
    "at_ctx_stream": [_vp, _PP],
    "at_ctx_set_stream": [_vp, _vp],
    "at_alloc": [_vp, _sz, _PP],
    "at_free": [_vp, _vp],
    "at_memcpy_h2d": [_vp, _vp, _vp, _sz],
    "at_memcpy_d2h": [_vp, _vp, _vp, _sz],
    "at_memset_zero": [_vp, _vp, _sz],
    "at_fp16_to_f32": [_vp, _vp, _vp, _i64],
    "at_q4_0_dequant": [_vp, _vp, _vp, _i64],
    "at_q8_0_dequant": [_vp, _vp, _vp, _i64],
    "at_q6_k_dequant": [_vp, _vp, _vp, _i64],
    "at_q4_0_dot": [_vp, _vp, _vp, _i64, _vp],
    "at_q8_0_dot": [_vp, _vp, _vp, _i64, _vp],
    "at_qmat_create": [_vp, _i, _i, _i64, _i64, _vp, _i, _PP],
    "at_qmat_create_ex": [_vp, _i, _i, _i, _i64, _i64, _vp, _i, _PP],
    "at_qmat_destroy": [_vp],
    "at_qmat_export": [_vp, _vp, _vp],
    "at_gemv": [_vp, _vp, _vp, _vp, _i],
    "at_gemv_t_static_scratch": [_vp, _vp, _vp, _vp, _i],
    "at_gemm_tc": [_vp, _vp, _vp, _vp, _i],
    "at_sgemv": [_vp, _vp, _vp, _vp, _i, _i],
    "at_sgemm": [_vp, _vp, _vp, _vp, _i, _i, _i],
    "at_rmsnorm": [_vp, _vp, _vp, _f, _i, _i],
    "at_softmax": [_vp, _vp, _i, _i],
    "at_rope": [_vp, _vp, _vp, _vp, _i, _i],
    "at_silu": [_vp, _vp, _i64],
    "at_model_create": [_vp, C.POINTER(ModelConfig), _PP],
    "at_model_set_tensor": [_vp, C.c_char_p, _i, _vp, _sz, _i],
    "at_model_finalize": [_vp],
    "at_model_load_gguf": [_vp, C.c_char_p, _i, _PP],
    "at_model_load_gguf_ex": [_vp, C.c_char_p, _i, _i, _i, _PP],
    "at_model_get_config": [_vp, C.POINTER(ModelConfig)],
    "at_model_destroy": [_vp],
    "at_model_forward_step": [_vp, _i, _i64, _vp],
    "at_model_forward_prompt": [_vp, _vp, _i],
    "at_model_forward_batch": [_vp, _vp, _vp, _i, _vp],
    "at_model_logits_device": [_vp, _PP],
    "at_model_argmax": [_vp, _i, _vp],
    "at_model_step_kernel": [_vp, _vp],
    "at_model_step_stamps": [_vp, _i, _i64, _vp, _i64, _vp],
    "at_model_generate": [_vp, _i, _i64, _i, _vp],
    "at_model_profile_step": [_vp, _i, _i64, _vp, _vp],
    "at_model_profile_batch": [_vp, _i, _vp, _vp, _vp, _vp],
    "at_model_sample": [_vp, _i, _vp, _vp],
    "at_model_generate_sampled": [_vp, _i, _vp, _vp, _i, _vp, _vp],
    "at_model_forward_prompt_slot": [_vp, _i, _vp, _i],
    "at_sched_create": [_vp, _PP],
    "at_sched_destroy": [_vp],
    "at_sched_submit": [_vp, _vp, _i, _i, _i, _vp, C.POINTER(C.c_int)],
    "at_sched_step": [_vp, C.POINTER(C.c_int)],
    "at_sched_result": [_vp, _i, _vp, _i, C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "at_model_kv_size": [_vp, _i, C.POINTER(C.c_int64)],
    "at_model_kv_read": [_vp, _i, _i, _i, _i64, _vp, _vp],
    "at_model_kv_reset": [_vp, _i],
    "at_model_kv_append": [_vp, _i, _i64, _i64, _vp, _vp],
    "at_model_kv_offset": [_vp, _i64, _i64, _i64, _i64, C.POINTER(C.c_int64)],
    "at_sample": [_vp, _i, _vp, _i, _f, _i, _f, _f, _i64, C.POINTER(C.c_int)],
    "at_tp_unique_id": [_vp],
    "at_ctx_create_tp": [_i, _i, _i, _vp, _PP],
    "at_tp_shard_region": [_vp, _i, _i, C.c_char_p, _vp],
}

_lib = None
_lock = threading.Lock()


def lib():
    """Loads the in-tree shared library once; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: run auratensor_b200.build.build() first")
            L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
            for name, args in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = C.c_int
            L.at_version.restype = C.c_char_p
            L.at_version.argtypes = []
            _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().at_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != AT_OK:
        raise _EXC.get(rc, AtError)(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
