"""Oracle: MLX-style affine group quantization of weights (test infrastructure only).

Nothing in the product path imports this module; tests, the smoke check and
the benchmark's CPU baseline use it as the checker.

Format (the one ``mx.quantize`` produces and ``mx.quantized_matmul`` /
``mx.gather_qmm`` consume, as called at
``mlx_flash_compress/layer_quantization.py:254`` and
``mlx_flash_compress/expert_streaming.py:230-241``):

* ``W[..., K]`` is split along its last axis into groups of ``group_size``.
* ``q`` is packed little-end first into uint32 words: element ``k`` sits at bit
  ``bits * (k % (32 // bits))`` of word ``k // (32 // bits)``.  This is the
  unpack order restated in NumPy at ``mixed_precision.py:150-171`` (view the
  word as little-endian bytes, low nibble first).
* dequantize: ``w = q * scale + bias`` (float32 multiply, then float32 add,
  then one rounding into the weight dtype) -- ``mixed_precision.py:161-171``.

Two per-group scale/bias rules (float32 arithmetic, n = 2**bits - 1):

``rule="mlx"`` (default) -- MLX's ``affine_quantize``, restated from the
published source of ml-explore/mlx (``mlx/ops.cpp`` ``affine_quantize`` and
its CPU kernel in ``mlx/backend/cpu/quantized.cpp``, releases 0.24-0.26; the
reference pins ``mlx>=0.24.0``, ``pyproject.toml:26``).  MLX is not
installable here, so the restatement is checked against hand-derived known
answers, not against MLX output:
  1. ``scale = max((max - min) / n, 1e-7)``;
  2. the edge is the group's larger-magnitude end: if ``|min| > |max|`` the
     edge is ``min`` and the scale stays positive, else the edge is ``max``
     and the scale is negated;
  3. ``q0 = rint(edge / scale)``; if ``q0 != 0`` then ``scale = edge / q0``
     and ``bias = edge`` (the edge, and zero, land exactly on the code grid),
     else ``bias = 0``;
  4. ``q = clip(rint((w - bias) / scale), 0, n)`` with the float32 scale and
     bias; only then are scale and bias rounded into the weight dtype.
  ``rint`` rounds half to even (MLX's ``round`` and ``std::rint``).

``rule="minmax"`` -- the rule the single-linear workload states: ``scale =
(max - min) / n`` rounded to the weight dtype, ``bias = min``, ``q`` computed
with the rounded scale; a group whose rounded scale is 0 gets ``q = 0`` so
that it dequantizes to exactly ``bias``.

Arithmetic is written with float32 NumPy operations so that each step is one
IEEE-754 rounding, matching the CUDA kernels' ``__fsub_rn``/``__fdiv_rn``/
``rintf``.
"""

import numpy as np

from .fp import round_to

SUPPORTED_BITS = (2, 4, 8)


def _check(bits, group_size, K):
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"bits must be one of {SUPPORTED_BITS}, got {bits}")
    if group_size <= 0 or K % group_size != 0:
        raise ValueError(f"last dimension {K} must be divisible by group_size {group_size}")


def quantize(w, group_size: int = 64, bits: int = 4, dtype: str = "bf16", rule: str = "mlx"):
    """Return ``(wq uint32, scales f32, biases f32)``; scales/biases hold ``dtype`` values."""
    w = np.asarray(w, dtype=np.float32)
    K = w.shape[-1]
    _check(bits, group_size, K)
    if rule not in ("mlx", "minmax"):
        raise ValueError(f"rule must be 'mlx' or 'minmax', got {rule!r}")
    lead = w.shape[:-1]
    g = w.reshape(*lead, K // group_size, group_size)
    n_bins = np.float32((1 << bits) - 1)
    wmax = g.max(axis=-1).astype(np.float32)
    wmin = g.min(axis=-1).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        if rule == "mlx":
            scale = np.maximum((wmax - wmin).astype(np.float32) / n_bins, np.float32(1e-7)).astype(np.float32)
            side = np.abs(wmin) > np.abs(wmax)
            scale = np.where(side, scale, -scale).astype(np.float32)
            edge = np.where(side, wmin, wmax).astype(np.float32)
            q0 = np.rint(edge / scale).astype(np.float32)
            nz = q0 != 0
            scale = np.where(nz, edge / np.where(nz, q0, np.float32(1)), scale).astype(np.float32)
            bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
            t = (g - bias[..., None]).astype(np.float32) / scale[..., None]
            q = np.clip(np.rint(t), 0, n_bins).astype(np.uint32)
            scale = round_to(scale, dtype).astype(np.float32)
            bias = round_to(bias, dtype).astype(np.float32)
        else:
            scale = round_to((wmax - wmin).astype(np.float32) / n_bins, dtype).astype(np.float32)
            bias = wmin.astype(np.float32)
            safe = np.where(scale == 0, np.float32(1), scale).astype(np.float32)
            t = (g - bias[..., None]).astype(np.float32) / safe[..., None]
            q = np.clip(np.rint(t), 0, n_bins)
            q = np.where((scale == 0)[..., None], 0, q).astype(np.uint32)
    q = q.reshape(*lead, K)
    per = 32 // bits
    qw = q.reshape(*lead, K // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    wq = np.bitwise_or.reduce(qw << shifts, axis=-1).astype(np.uint32)
    return wq, scale, bias


def unpack(wq, bits: int = 4) -> np.ndarray:
    """uint32 words -> integer codes (uint32), element order k = word*per + slot."""
    wq = np.asarray(wq, dtype=np.uint32)
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    q = (wq[..., None] >> shifts) & mask
    return q.reshape(*wq.shape[:-1], wq.shape[-1] * per)


def dequantize_f32(wq, scales, biases, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """``q*scale + bias`` in float32 (one rounding for the product, one for the sum)."""
    q = unpack(wq, bits).astype(np.float32)
    K = q.shape[-1]
    s = np.repeat(np.asarray(scales, np.float32), group_size, axis=-1)[..., :K]
    b = np.repeat(np.asarray(biases, np.float32), group_size, axis=-1)[..., :K]
    return (q * s).astype(np.float32) + b


def dequantize(wq, scales, biases, group_size: int = 64, bits: int = 4, dtype: str = "bf16"):
    """Dequantized weights rounded into ``dtype`` (returned as float32)."""
    return round_to(dequantize_f32(wq, scales, biases, group_size, bits), dtype)


def quantized_matmul(x, wq, scales, biases, transpose: bool = True, group_size: int = 64,
                     bits: int = 4, out_dtype: str = "bf16"):
    """``x @ dequant(W).T`` accumulated in float64 from the exact float32 dequant."""
    if not transpose:
        raise ValueError("only transpose=True is part of this path")
    W = dequantize_f32(wq, scales, biases, group_size, bits).astype(np.float64)
    y = np.asarray(x, np.float64) @ np.swapaxes(W, -1, -2)
    return round_to(y.astype(np.float32), out_dtype)


def gather_qmm(x, wq, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size: int = 64, bits: int = 4, out_dtype: str = "bf16"):
    """Batched gather of ``x`` rows and stacked quantized matrices, then qmm.

    ``x``: ``[..., M, K]``; ``wq``: ``[E, N, K*bits/32]`` (scales/biases ``[E, N, K/gs]``).
    The batch shape is the broadcast of the index arrays with the batch dims of
    whichever operand is not indexed; result ``[*batch, M, N]``.
    """
    if not transpose:
        raise ValueError("only transpose=True is part of this path")
    x = np.asarray(x, np.float32)
    wq = np.asarray(wq, np.uint32)
    xb = x.shape[:-2]
    wb = wq.shape[:-2]
    M, K = x.shape[-2:]
    N = wq.shape[-2]
    x_flat = x.reshape(-1, M, K)
    w_flat = wq.reshape(-1, *wq.shape[-2:])
    s_flat = np.asarray(scales, np.float32).reshape(-1, *np.shape(scales)[-2:])
    b_flat = np.asarray(biases, np.float32).reshape(-1, *np.shape(biases)[-2:])
    if lhs_indices is None:
        lhs = np.arange(int(np.prod(xb)) if xb else 1).reshape(xb if xb else ())
    else:
        lhs = np.asarray(lhs_indices)
    if rhs_indices is None:
        rhs = np.arange(int(np.prod(wb)) if wb else 1).reshape(wb if wb else ())
    else:
        rhs = np.asarray(rhs_indices)
    lhs, rhs = np.broadcast_arrays(lhs, rhs)
    out = np.zeros((*lhs.shape, M, N), np.float32)
    W_cache = {}
    for idx in np.ndindex(*lhs.shape):
        e = int(rhs[idx])
        if e not in W_cache:
            W_cache[e] = dequantize_f32(w_flat[e], s_flat[e], b_flat[e], group_size, bits).astype(np.float64)
        y = x_flat[int(lhs[idx])].astype(np.float64) @ W_cache[e].T
        out[idx] = y
    return round_to(out, out_dtype)
