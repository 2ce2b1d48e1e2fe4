"""``CUDABackend``: the reference's ``smallm::Backend`` interface
(include/smallm/backend/common/backend.h:12-38) on the B200.

Same six operations, same argument meaning, host numpy arrays in and out
(operations the reference performs in place -- softmax, silu, rope -- modify
the array in place here too).  Errors raise ``SmallmError`` where the
reference throws.  ``matmul_quantized`` keeps a device copy of each weight
matrix keyed by the host buffer's address, as the reference hands the
backend the same mmap pointer for a weight on every call.

Device-resident operands (``QMatrix`` + ``gemv``) run the same kernels on
data that stays in HBM.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check, lib


def _f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


class CUDABackend:
    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().smallm_ctx_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        self._keep = {}

    def close(self):
        if getattr(self, "h", None):
            lib().smallm_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().smallm_ctx_stream(self.h) or 0

    def synchronize(self):
        check(lib().smallm_ctx_synchronize(self.h))

    # ---- Backend (backend.h:17-37) ----
    def matmul(self, W, x, rows: int, cols: int) -> np.ndarray:
        W = _f32(W)
        x = _f32(x)
        y = np.empty(rows, dtype=np.float32)
        self._keep[W.ctypes.data] = W
        check(lib().smallm_backend_matmul(self.h, W.ctypes.data, x.ctypes.data, rows, cols, y.ctypes.data))
        return y

    def matmul_quantized(self, W, type_: int, x, rows: int, cols: int) -> np.ndarray:
        W = _u8(W) if not (isinstance(W, np.ndarray) and W.dtype == np.uint8 and W.flags.c_contiguous) else W
        x = _f32(x)
        y = np.empty(rows, dtype=np.float32)
        self._keep[W.ctypes.data] = W  # the device copy is keyed by this address
        check(lib().smallm_backend_matmul_quantized(self.h, W.ctypes.data, type_, x.ctypes.data, rows, cols,
                                                    y.ctypes.data))
        return y

    def rmsnorm(self, x, weight, size: int, eps: float) -> np.ndarray:
        x = _f32(x)
        w = _f32(weight)
        y = np.empty(size, dtype=np.float32)
        check(lib().smallm_backend_rmsnorm(self.h, x.ctypes.data, w.ctypes.data, size, eps, y.ctypes.data))
        return y

    def softmax(self, x: np.ndarray, size: int | None = None) -> np.ndarray:
        assert x.dtype == np.float32 and x.flags.c_contiguous
        check(lib().smallm_backend_softmax(self.h, x.ctypes.data, x.size if size is None else size))
        return x

    def silu(self, x: np.ndarray, size: int | None = None) -> np.ndarray:
        assert x.dtype == np.float32 and x.flags.c_contiguous
        check(lib().smallm_backend_silu(self.h, x.ctypes.data, x.size if size is None else size))
        return x

    def rope(self, x: np.ndarray, n_heads: int, head_dim: int, pos: int, freq_base: float) -> np.ndarray:
        assert x.dtype == np.float32 and x.flags.c_contiguous
        check(lib().smallm_backend_rope(self.h, x.ctypes.data, n_heads, head_dim, pos, freq_base))
        return x

    def clear_weights(self):
        check(lib().smallm_ctx_clear_weights(self.h))
        self._keep.clear()

    # ---- extras ----
    def dequantize(self, type_: int, raw, count: int) -> np.ndarray:
        raw = _u8(raw)
        out = np.empty(count, dtype=np.float32)
        check(lib().smallm_dequantize(self.h, type_, raw.ctypes.data, count, out.ctypes.data))
        return out

    def upload(self, W, type_: int, rows: int, cols: int) -> "QMatrix":
        return QMatrix(self, W, type_, rows, cols)


class QMatrix:
    """A weight matrix repacked into HBM (smallm_qmatrix_*)."""

    def __init__(self, be: CUDABackend, W, type_: int, rows: int, cols: int):
        W = _u8(W)
        h = ctypes.c_void_p()
        check(lib().smallm_qmatrix_upload(be.h, W.ctypes.data, type_, rows, cols, ctypes.byref(h)))
        self.h, self.be, self.type, self.rows, self.cols = h, be, type_, rows, cols

    def bytes(self) -> tuple[int, int]:
        g, d = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().smallm_qmatrix_bytes(self.h, ctypes.byref(g), ctypes.byref(d)))
        return g.value, d.value

    def gemv(self, x_dev: int, y_dev: int, stream: int | None = None):
        check(lib().smallm_gemv(self.be.h, self.h, x_dev, y_dev, stream))

    def dequantize_to(self, y_dev: int, stream: int | None = None):
        check(lib().smallm_qmatrix_dequantize(self.be.h, self.h, y_dev, stream))

    def free(self):
        if getattr(self, "h", None):
            lib().smallm_qmatrix_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
