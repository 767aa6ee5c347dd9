"""Oracle: Q4_0 dequant-GEMV through the C restatement ``q4_0_gemv.c``
(``mlx_flash_compress/kernels/flash_dequant.metal:19-49``); test
infrastructure only.  Builds the C library on first use."""

import ctypes

import numpy as np

from . import _cbuild

_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(_cbuild.build())
        _lib.q4_0_gemv.restype = None
        _lib.q4_0_gemv.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_uint32] * 3
    return _lib


def gemv(weights, scales_f16, x, group_size: int = 32) -> np.ndarray:
    """``weights`` uint8 [M, N/2], ``scales_f16`` float16 [M, N/gs], ``x`` fp32 [N] -> fp32 [M]."""
    w = np.ascontiguousarray(weights, np.uint8)
    s = np.ascontiguousarray(scales_f16, np.float16).view(np.uint16)
    xv = np.ascontiguousarray(x, np.float32)
    M, N = w.shape[0], w.shape[1] * 2
    y = np.empty(M, np.float32)
    _load().q4_0_gemv(w.ctypes.data, s.ctypes.data, xv.ctypes.data, y.ctypes.data, M, N, group_size)
    return y


def gemv_numpy(weights, scales_f16, x, group_size: int = 32) -> np.ndarray:
    """float64 reference of the same sum (no accumulation-order effects)."""
    w = np.asarray(weights, np.uint8)
    codes = np.empty((w.shape[0], w.shape[1] * 2), np.float64)
    codes[:, 0::2] = w & 0xF
    codes[:, 1::2] = w >> 4
    s = np.repeat(np.asarray(scales_f16, np.float64), group_size, axis=1)
    return ((codes - 8.0) * s) @ np.asarray(x, np.float64)
