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


def route(x, wr, top_k, renorm=True, bias=None, gating="softmax", skip_threshold=0.0):
    """Top-k routing; ``wr`` is [H, E].  Returns (inds [T,k], scores [T,k]).

    ``gating="softmax"``: ``softmax(x.wr + bias)`` (``expert_streaming.py:440``);
    ``"sigmoid"``: ``sigmoid`` per expert.  Ties in the gate value are broken
    by the lower expert id; slots are in descending gate order.  With
    ``skip_threshold > 0``, the LExI mask (``expert_streaming.py:451-457``):
    slot 0 is kept, slot j >= 1 is zeroed where ``top1 > skip * score_j``;
    then ``renorm`` divides by the sum where it is positive (``:459-460``).
    """
    logits = np.asarray(x, np.float64) @ np.asarray(wr, np.float64)
    if bias is not None:
        logits = logits + np.asarray(bias, np.float64)
    if gating == "sigmoid":
        g = 1.0 / (1.0 + np.exp(-logits))
    else:
        logits = logits - logits.max(axis=-1, keepdims=True)
        g = np.exp(logits)
        g /= g.sum(axis=-1, keepdims=True)
    order = np.lexsort((np.broadcast_to(np.arange(g.shape[-1]), g.shape), -g), axis=-1)
    inds = order[..., :top_k]
    scores = np.take_along_axis(g, inds, axis=-1)
    if skip_threshold > 0 and top_k > 1:
        keep = ~(scores[..., :1] > skip_threshold * scores)
        keep[..., 0] = True
        scores = scores * keep
    if renorm:
        tot = scores.sum(axis=-1, keepdims=True)
        scores = np.where(tot > 0, scores / np.where(tot > 0, tot, 1), scores)
    return inds.astype(np.int32), scores


def shared_expert(x, gate, up, down, gate_weight=None, group_size=64, bits=4):
    """``sigmoid(x . gate_weight) * down(silu(gate x) * up x)`` for one dense
    SwiGLU expert (``expert_streaming.py:466-470``); ``gate``/``up``/``down``
    are (wq, scales, biases) of single matrices.  Returns [T, H] float64."""
    x = np.asarray(x, np.float64)
    Wg, Wu, Wd = (affine.dequantize_f32(*t, group_size, bits).astype(np.float64) for t in (gate, up, down))
    y = (silu(x @ Wg.T) * (x @ Wu.T)) @ Wd.T
    if gate_weight is not None:
        y = y / (1.0 + np.exp(-(x @ np.asarray(gate_weight, np.float64).reshape(-1, 1))))
    return y


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
