"""Oracle: the reference's symmetric absmax KV quantizer (test infrastructure only).

Restates ``quantize_tensor`` and ``dequantize_tensor`` from
``mlx_flash_compress/quantized_kv_cache.py:68-156`` and ``:159-234`` step by
step.  Every arithmetic step of the reference is an MLX op on an array of the
input dtype, so each is restated as "float32 op, then round into that dtype"
(``round_to``): this is how MLX evaluates bf16/fp16 element-wise ops, and it is
what makes the packed bytes bit-exact.

Format (per row of the last axis ``D``):
  ``gs = min(group_size, D)``; the row is zero-padded to a multiple of ``gs``;
  ``max_int = 2**(bits-1) - 1``; ``scale = absmax / max_int`` (0 -> 1);
  ``code = clip(round(x / scale), -max_int, max_int) + max_int`` as uint8;
  8-bit: one code per byte; 4-bit: byte ``i`` = ``code[2i] << 4 | code[2i+1]``;
  2-bit: byte ``i`` = ``c[4i]<<6 | c[4i+1]<<4 | c[4i+2]<<2 | c[4i+3]``;
  odd tails of the packing are padded with code 0.  Scales are float32, the
  "zeros" output is all 0.  Dequantize: ``(code - max_int) * scale`` in float32.
"""

import numpy as np

from .fp import round_to


def _check_bits(bits):
    if bits not in (2, 4, 8):
        raise ValueError(f"bits must be 2, 4, or 8, got {bits}")


def packed_len(D: int, bits: int, group_size: int) -> int:
    """Bytes per row for a last axis of length ``D`` (quantized_kv_cache.py:94-154)."""
    gs = min(group_size, D)
    dp = D if D % gs == 0 else D + gs - D % gs
    if bits == 8:
        return dp
    if bits == 4:
        return (dp + 1) // 2
    return (dp + 3) // 4


def num_groups(D: int, group_size: int) -> int:
    gs = min(group_size, D)
    dp = D if D % gs == 0 else D + gs - D % gs
    return dp // gs


def quantize_tensor(x, bits: int, group_size: int = 64, dtype: str = "f32"):
    """Return ``(packed uint8, scales f32, zeros f32)`` exactly as the reference does."""
    _check_bits(bits)
    if group_size <= 0:
        raise ValueError(f"group_size must be positive, got {group_size}")
    x = np.asarray(x, dtype=np.float32)
    shape = x.shape
    if not shape or shape[-1] == 0:
        e = np.zeros((0,), np.float32)
        return np.zeros((0,), np.uint8), e, e.copy()
    D = shape[-1]
    gs = min(group_size, D)
    if D % gs != 0:
        pad = gs - D % gs
        x = np.concatenate([x, np.zeros((*shape[:-1], pad), np.float32)], axis=-1)
        D = x.shape[-1]
    lead = list(shape[:-1])
    ng = D // gs
    xg = x.reshape(*lead, ng, gs)
    max_int = (1 << (bits - 1)) - 1
    gmax = np.abs(xg).max(axis=-1, keepdims=True)
    scales = round_to(gmax / np.float32(max_int), dtype)
    scales = np.where(scales == 0, np.float32(1), scales).astype(np.float32)
    xs = round_to(xg / scales, dtype)
    xq = round_to(np.rint(xs), dtype)
    xq = np.clip(xq, -max_int, max_int)
    scales_out = scales[..., 0].astype(np.float32)
    zeros_out = np.zeros_like(scales_out)
    xu = round_to(xq + np.float32(max_int), dtype).astype(np.uint8)
    flat = xu.reshape(*lead, ng * gs)
    if bits == 8:
        packed = flat
    elif bits == 4:
        if flat.shape[-1] % 2:
            flat = np.concatenate([flat, np.zeros((*lead, 1), np.uint8)], axis=-1)
        packed = ((flat[..., 0::2] << 4) | (flat[..., 1::2] & 0x0F)).astype(np.uint8)
    else:
        r = flat.shape[-1] % 4
        if r:
            flat = np.concatenate([flat, np.zeros((*lead, 4 - r), np.uint8)], axis=-1)
        packed = ((flat[..., 0::4] << 6) | ((flat[..., 1::4] & 3) << 4)
                  | ((flat[..., 2::4] & 3) << 2) | (flat[..., 3::4] & 3)).astype(np.uint8)
    return packed, scales_out, zeros_out


def dequantize_tensor(quantized, scales, zeros, bits: int, original_shape, group_size: int = 64):
    """float32 reconstruction exactly as ``dequantize_tensor`` computes it."""
    _check_bits(bits)
    original_shape = tuple(original_shape)
    if not original_shape or original_shape[-1] == 0:
        return np.zeros(original_shape, np.float32)
    q = np.asarray(quantized, np.uint8)
    max_int = (1 << (bits - 1)) - 1
    lead = list(original_shape[:-1])
    D = original_shape[-1]
    gs = min(group_size, D)
    if bits == 8:
        xu = q
    elif bits == 4:
        xu = np.stack([(q >> 4) & 0x0F, q & 0x0F], axis=-1).reshape(*lead, -1)
    else:
        xu = np.stack([(q >> 6) & 3, (q >> 4) & 3, (q >> 2) & 3, q & 3], axis=-1).reshape(*lead, -1)
    xs = xu.astype(np.float32) - np.float32(max_int)
    dp = D if D % gs == 0 else D + gs - D % gs
    xs = xs[..., :dp]
    ng = dp // gs
    xg = xs.reshape(*lead, ng, gs)
    se = np.asarray(scales, np.float32)[..., :ng].reshape(*lead, ng, 1)
    return (xg * se).reshape(*lead, dp)[..., :D].astype(np.float32)
