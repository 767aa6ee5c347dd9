"""Floating-point helpers for the CPU oracle (test infrastructure only).

NumPy has no bfloat16, so bf16 values are carried as float32 arrays whose
values are exactly representable in bf16.  ``round_bf16`` performs IEEE
round-to-nearest-even from float32 to bf16 (NaN kept quiet), which is what
MLX's ``astype(bfloat16)`` and CUDA's ``__float2bfloat16_rn`` do.
"""

import numpy as np


def round_bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (ties to even)."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, (u.astype(np.uint32) | 0x00400000) & 0xFFFF0000, r).astype(np.uint32)
    return r.view(np.float32).reshape(a.shape)


def round_f16(x) -> np.ndarray:
    """Round float32 values to the nearest fp16 value, returned as float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values into ``dtype`` ("bf16", "f16" or "f32")."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of bf16-representable float32 values."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    """float32 values from uint16 bf16 bit patterns."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def allclose_report(got, want, rtol=1e-2, atol=2e-2) -> tuple:
    """(ok, max_abs_err, worst_index) for |got-want| <= atol + rtol*|want|."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = err > bound
    worst = int(np.argmax(err - bound)) if err.size else 0
    return (not bad.any()), (float(err.max()) if err.size else 0.0), worst
