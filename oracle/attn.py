"""Oracle: GQA decode attention over dequantized K/V (test infrastructure only).

The reference has no attention kernel over quantized KV: ``get_keys_values``
(``mlx_flash_compress/quantized_kv_cache.py:311-358``) dequantizes every chunk
to float32 and the caller runs ordinary attention.  This restates that
consumer: dequantize (``oracle.kv_sym``), then softmax(q.K^T * scale).V in
float64, query head ``h`` reading KV head ``h // (Hq/Hkv)``.  It also returns
the head-mean of the attention row that ``kv_compression.py:84-106`` scores.
"""

import numpy as np


def decode_attention(q, keys, values, softmax_scale=None):
    """``q``: [B, Hq, D]; ``keys``/``values``: list of [S_b, Hkv, D] arrays.

    Returns ``(out [B, Hq, D] float32, head_mean_probs list of [S_b])``.
    """
    q = np.asarray(q, np.float64)
    B, Hq, D = q.shape
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    out = np.zeros((B, Hq, D), np.float64)
    means = []
    for b in range(B):
        k = np.asarray(keys[b], np.float64)
        v = np.asarray(values[b], np.float64)
        S, Hkv, _ = k.shape
        G = Hq // Hkv
        probs = np.zeros((Hq, S))
        for h in range(Hq):
            kh = k[:, h // G, :]
            s = kh @ q[b, h] * softmax_scale
            if S == 0:
                continue
            s = s - s.max()
            p = np.exp(s)
            p /= p.sum()
            probs[h] = p
            out[b, h] = p @ v[:, h // G, :]
        means.append(probs.mean(axis=0) if S else np.zeros(0))
    return out.astype(np.float32), means
