"""Oracle: per-tensor symmetric fake quantization used by layer-sensitivity
profiling (``mlx_flash_compress/layer_quantization.py:461-494``); test
infrastructure only.

MLX evaluation order, with the dtype rules of ``mlx.core``: ``abs_max =
max(|w|)`` in w's dtype; ``scale = abs_max / qmax`` rounded to w's dtype
(a Python scalar takes the array's dtype); ``mx.maximum(scale,
mx.array(1e-10))`` promotes to float32; ``w / scale``, ``round`` (half to
even), ``clip`` and ``* scale`` are float32.
"""

import numpy as np

from .fp import round_to


def fake_quantize_sym(w, bits: int = 4, dtype: str = "bf16"):
    """``w``: float32 values exact in ``dtype`` ("bf16", "f16" or "f32").  Returns (out f32, absmax)."""
    w = np.asarray(w, np.float32)
    qmax, qmin = (7.0, -8.0) if bits <= 4 else (127.0, -128.0)
    amax = np.float32(np.abs(w).max()) if w.size else np.float32(0)
    scale = np.float32(amax) / np.float32(qmax)
    if dtype != "f32":
        scale = round_to(np.asarray([scale], np.float32), dtype)[0]
    scale = np.maximum(np.float32(scale), np.float32(1e-10))
    q = np.clip(np.rint(w / scale), qmin, qmax).astype(np.float32)
    return (q * scale).astype(np.float32), amax
