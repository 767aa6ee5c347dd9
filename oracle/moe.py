"""Oracle: router + routed SwiGLU experts (test infrastructure only).

Restates the MoE block as MLX-Flash drives it:
``gates = softmax(x.Wr)``, top-k, optional renormalisation
(``mlx_flash_compress/expert_streaming.py:439-472``); per (token, k):
``silu(x.Wg^T) * (x.Wu^T)`` then ``.Wd^T`` with each projection an affine
quantized ``gather_qmm`` (``expert_streaming.py:224-241``); combine
``sum_k score_k * y_k`` (``kernels/ops.py:111-148``).  float64 throughout.
"""

import numpy as np

from . import affine


def route(x, wr, top_k, renorm=True):
    """Softmax top-k routing; ``wr`` is [H, E].  Returns (inds [T,k], scores [T,k]).

    Ties in the gate value are broken by the lower expert id.
    """
    logits = np.asarray(x, np.float64) @ np.asarray(wr, np.float64)
    logits = logits - logits.max(axis=-1, keepdims=True)
    g = np.exp(logits)
    g /= g.sum(axis=-1, keepdims=True)
    order = np.lexsort((np.broadcast_to(np.arange(g.shape[-1]), g.shape), -g), axis=-1)
    inds = order[..., :top_k]
    scores = np.take_along_axis(g, inds, axis=-1)
    if renorm:
        scores = scores / scores.sum(axis=-1, keepdims=True)
    return inds.astype(np.int32), scores


def silu(v):
    return v / (1.0 + np.exp(-v))


def expert_mlp(x, inds, scores, gate, up, down, group_size=64, bits=4):
    """``gate/up/down`` are (wq, scales, biases) stacked over experts.

    Returns (y [T, H] combined, h [T, k, I] SwiGLU activations, yk [T, k, H]).
    """
    x = np.asarray(x, np.float64)
    T, k = inds.shape
    cache = {}

    def W(which, e):
        key = (which, e)
        if key not in cache:
            wq, s, b = (gate, up, down)[which]
            cache[key] = affine.dequantize_f32(wq[e], s[e], b[e], group_size, bits).astype(np.float64)
        return cache[key]

    H = x.shape[-1]
    I = W(0, int(inds[0, 0])).shape[0]
    h = np.zeros((T, k, I))
    yk = np.zeros((T, k, H))
    for t in range(T):
        for j in range(k):
            e = int(inds[t, j])
            g = W(0, e) @ x[t]
            u = W(1, e) @ x[t]
            h[t, j] = silu(g) * u
            yk[t, j] = W(2, e) @ h[t, j]
    y = (yk * np.asarray(scores, np.float64)[..., None]).sum(axis=1)
    return y, h, yk
