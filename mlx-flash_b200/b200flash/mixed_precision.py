"""Drop-in for the 2-bit path of ``mlx_flash_compress/mixed_precision.py``.

``requantize_4bit_to_2bit`` / ``dequantize_2bit`` (``:130-255``) on the GPU,
bit-exact with the NumPy reference: per group of codes ``v = nib*s + b``,
``crumb = clip(rint((v - min) / range * 3), 0, 3)`` (``range`` floored at
1e-10), fp16 ``scale = range / 3`` and ``bias = min``, crumbs packed
LSB-first four to a byte across the row.
"""

import torch

from ._capi import call, ptr, require_cuda, stream_of

_DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def requantize_4bit_to_2bit(weight_uint32: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                            group_size: int = 128):
    """Returns ``(packed uint8 [rows, 2*cols_u32], scales fp16, biases fp16, metadata)``.

    As in the reference, the group width comes from the ``scales`` shape
    (``8*cols_u32 / n_groups``); ``group_size`` is accepted for signature
    compatibility and not used.
    """
    dev = require_cuda(weight_uint32, scales, biases)
    if weight_uint32.dtype not in (torch.uint32, torch.int32):
        raise ValueError("weight_uint32 must be a 32-bit integer tensor")
    if scales.dtype not in _DT or biases.dtype != scales.dtype:
        raise ValueError("scales and biases must share a float dtype")
    wq = weight_uint32.contiguous()
    rows, cols = wq.shape
    ng = scales.shape[1]
    packed = torch.empty(rows, 2 * cols, dtype=torch.uint8, device=dev)
    s2 = torch.empty(rows, ng, dtype=torch.float16, device=dev)
    b2 = torch.empty_like(s2)
    call("b2f_requant_4to2", ptr(wq), rows, cols, ptr(scales.contiguous()), ptr(biases.contiguous()),
         _DT[scales.dtype], ng, ptr(packed), ptr(s2), ptr(b2), stream_of(dev))
    meta = {
        "original_shape": tuple(wq.shape),
        "packed_shape": tuple(packed.shape),
        "n_groups": ng,
        "weights_per_group": cols * 8 // ng,
        "original_bytes": wq.numel() * 4 + scales.numel() * scales.element_size() * 2,
        "packed_bytes": packed.numel() + s2.numel() * 4,
    }
    meta["ratio"] = meta["original_bytes"] / meta["packed_bytes"] if meta["packed_bytes"] else 0
    return packed, s2, b2, meta


def dequantize_2bit(packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                    n_values_per_row: int) -> torch.Tensor:
    """fp32 ``[rows, n_values_per_row] = crumb * scale + bias`` (mixed_precision.py:219-245)."""
    dev = require_cuda(packed, scales, biases)
    if scales.dtype != torch.float16 or biases.dtype != torch.float16:
        raise ValueError("2-bit scales/biases are fp16")
    p = packed.contiguous()
    rows = p.shape[0]
    out = torch.empty(rows, n_values_per_row, dtype=torch.float32, device=dev)
    call("b2f_dequant_2bit", ptr(p), p.shape[1], ptr(scales.contiguous()), ptr(biases.contiguous()),
         scales.shape[1], rows, n_values_per_row, ptr(out), stream_of(dev))
    return out
