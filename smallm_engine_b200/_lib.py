"""ctypes binding of libsmallm_cuda.so (the C ABI of include/smallm_cuda.h).

There is no CPU fallback: if the library is missing or cannot be loaded,
``lib()`` raises, and every call on a machine without an sm_100 GPU returns
SMALLM_ERR_CUDA, which the wrappers turn into ``SmallmError``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
# SMALLM_CUDA_LIB points at another build of the same library (e.g. a variant)
LIB_PATH = Path(os.environ.get("SMALLM_CUDA_LIB", PKG / "lib" / "libsmallm_cuda.so"))
HEADER = PKG.parent / "include" / "smallm_cuda.h"

OK = 0
ERR_INVALID, ERR_UNSUPPORTED_TYPE, ERR_CUDA, ERR_IO, ERR_FORMAT, ERR_NCCL, ERR_RANGE = 1, 2, 3, 4, 5, 6, 7
ERROR_NAMES = {1: "INVALID", 2: "UNSUPPORTED_TYPE", 3: "CUDA", 4: "IO", 5: "FORMAT", 6: "NCCL", 7: "RANGE"}


class SmallmError(RuntimeError):
    """A failed C-ABI call; ``code`` is the SMALLM_ERR_* value.  The reference
    raises std::runtime_error at the same points."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{ERROR_NAMES.get(code, code)}] {msg}")
        self.code = code


class ModelOpts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_ctx", ctypes.c_uint32), ("tp_rank", ctypes.c_int),
                ("tp_size", ctypes.c_int), ("nccl_id", ctypes.c_void_p), ("flags", ctypes.c_uint32)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("arch", ctypes.c_char * 16),
                ("n_layers", ctypes.c_uint32), ("embd", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("n_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("context_length", ctypes.c_uint32), ("max_ctx", ctypes.c_uint32),
                ("rope_freq_base", ctypes.c_float), ("rms_eps", ctypes.c_float),
                ("weight_bytes_per_token", ctypes.c_uint64), ("device_bytes", ctypes.c_uint64),
                ("step_launches", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_I = ctypes.c_int

# name -> (restype, argtypes)
SIGNATURES = {
    "smallm_last_error": (ctypes.c_char_p, []),
    "smallm_version": (_I, []),
    "smallm_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "smallm_ctx_destroy": (_I, [_P]),
    "smallm_ctx_stream": (_P, [_P]),
    "smallm_ctx_synchronize": (_I, [_P]),
    "smallm_backend_matmul": (_I, [_P, _P, _P, _U32, _U32, _P]),
    "smallm_backend_matmul_quantized": (_I, [_P, _P, _U32, _P, _U32, _U32, _P]),
    "smallm_backend_rmsnorm": (_I, [_P, _P, _P, _U32, ctypes.c_float, _P]),
    "smallm_backend_softmax": (_I, [_P, _P, _U32]),
    "smallm_backend_silu": (_I, [_P, _P, _U32]),
    "smallm_backend_rope": (_I, [_P, _P, _U32, _U32, _U32, ctypes.c_float]),
    "smallm_ctx_clear_weights": (_I, [_P]),
    "smallm_qmatrix_upload": (_I, [_P, _P, _U32, _U32, _U32, ctypes.POINTER(_P)]),
    "smallm_qmatrix_free": (_I, [_P]),
    "smallm_qmatrix_bytes": (_I, [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "smallm_gemv": (_I, [_P, _P, _P, _P, _P]),
    "smallm_gemm_f16": (_I, [_P, _P, _P, _U32, _U32, _U32, _P, _U32, _P]),
    "smallm_gemv_residual_sum": (_I, [_P, _P, _P, _P, _U32, _P, _P, _P, ctypes.c_float, _P, _P, _P]),
    "smallm_ctx_device_errors": (_I, [_P, ctypes.POINTER(_U32), ctypes.c_int]),
    "smallm_qmatrix_dequantize": (_I, [_P, _P, _P, _P]),
    "smallm_dequantize": (_I, [_P, _U32, _P, ctypes.c_uint64, _P]),
    "smallm_attention_noalloc": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _P, _P]),
    "smallm_sample": (_I, [_P, _P, _U32, _U32, _U32, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                           ctypes.POINTER(_U32)]),
    "smallm_model_sample": (_I, [_P, _U32, _U32, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                 ctypes.POINTER(_U32)]),
    "smallm_model_prefill": (_I, [_P, _P, _U32, _U32, _P, ctypes.POINTER(_U32), _U32]),
    "smallm_model_load": (_I, [ctypes.c_char_p, ctypes.POINTER(ModelOpts), ctypes.POINTER(_P)]),
    "smallm_model_free": (_I, [_P]),
    "smallm_model_get_info": (_I, [_P, ctypes.POINTER(ModelInfo)]),
    "smallm_model_stream": (_P, [_P]),
    "smallm_model_forward": (_I, [_P, _U32, _U32, _P, ctypes.POINTER(_U32)]),
    "smallm_model_reset_cache": (_I, [_P]),
    "smallm_model_truncate_cache": (_I, [_P, _U32]),
    "smallm_model_cached_length": (_U32, [_P]),
    "smallm_model_decode_greedy_async": (_I, [_P, _U32, _U32, _U32]),
    "smallm_model_decode_ids": (_I, [_P, _P, _U32]),
    "smallm_model_logits_device": (_P, [_P]),
    "smallm_model_trace_step": (_I, [_P, _U32, _U32, _P, _U32, ctypes.POINTER(_U32)]),
    "smallm_nccl_unique_id": (_I, [_P]),
    "smallm_host_alloc": (_I, [ctypes.c_size_t, ctypes.POINTER(_P)]),
    "smallm_host_free": (_I, [_P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load the CUDA backend library (built in-tree by
    ``python -m smallm_engine_b200.build``); raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m smallm_engine_b200.build` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        raise SmallmError(rc, lib().smallm_last_error().decode(errors="replace"))


def declared_symbols() -> list[str]:
    """Function names declared in include/smallm_cuda.h."""
    import re
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(smallm_[a-z0-9_]+)\s*\(", text)))
