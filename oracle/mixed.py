"""Oracle: 4-bit -> 2-bit expert requantization (test infrastructure only).

Restates ``requantize_4bit_to_2bit`` and ``dequantize_2bit`` from
``mlx_flash_compress/mixed_precision.py:130-255``, but unpacks the 4-bit words
with ``oracle.affine.unpack`` so that agreement with the reference pins the
affine unpack order.  Per group: float values ``q*s+b`` (float32), min/max,
``range<1e-10 -> 1e-10``, ``crumb = clip(rint((v-min)/range*3), 0, 3)``, fp16
``scale=range/3``, fp16 ``bias=min``; crumbs packed LSB-first, 4 per byte
(``mixed_precision.py:212-216``).
"""

import numpy as np

from . import affine


def requantize_4bit_to_2bit(wq, scales, biases, group_size: int = 64):
    wq = np.asarray(wq, np.uint32)
    rows = wq.shape[0]
    nib = affine.unpack(wq, 4).astype(np.float32)
    s = np.asarray(scales, np.float32)
    b = np.asarray(biases, np.float32)
    ng = s.shape[1]
    wpg = nib.shape[1] // ng
    vals = (nib * np.repeat(s, wpg, axis=1)) + np.repeat(b, wpg, axis=1)
    g = vals.reshape(rows, ng, wpg)
    gmin = g.min(axis=2, keepdims=True)
    gmax = g.max(axis=2, keepdims=True)
    rng = gmax - gmin
    rng = np.where(rng < 1e-10, np.float32(1e-10), rng).astype(np.float32)
    norm = (g - gmin) / rng * np.float32(3.0)
    crumbs = np.clip(np.rint(norm), 0, 3).astype(np.uint8).reshape(rows, ng * wpg)
    new_s = (rng[..., 0] / np.float32(3.0)).astype(np.float16)
    new_b = gmin[..., 0].astype(np.float16)
    n = crumbs.shape[1]
    pad = (-n) % 4
    if pad:
        crumbs = np.concatenate([crumbs, np.zeros((rows, pad), np.uint8)], axis=1)
    c4 = crumbs.reshape(rows, -1, 4)
    packed = (c4[..., 0] | (c4[..., 1] << 2) | (c4[..., 2] << 4) | (c4[..., 3] << 6)).astype(np.uint8)
    return packed, new_s, new_b


def dequantize_2bit(packed, scales, biases, n_values_per_row: int):
    p = np.asarray(packed, np.uint8)
    rows = p.shape[0]
    shifts = np.array([0, 2, 4, 6], np.uint8)
    crumbs = ((p[..., None] >> shifts) & 3).reshape(rows, -1)[:, :n_values_per_row]
    s = np.asarray(scales, np.float32)
    b = np.asarray(biases, np.float32)
    wpg = n_values_per_row // s.shape[1]
    return crumbs.astype(np.float32) * np.repeat(s, wpg, axis=1)[:, :n_values_per_row] \
        + np.repeat(b, wpg, axis=1)[:, :n_values_per_row]
