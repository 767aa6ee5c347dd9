"""Oracle: one decode step of the Qwen3-MoE-shaped decoder (test infrastructure only).

Built from the other oracle pieces; activations are rounded to bf16 at the
same points the GPU pipeline stores them (residual stream, normed inputs,
projections, q/k after norm and rotary, attention output, SwiGLU output,
expert outputs), every dot product is accumulated in float64.

Model: RMSNorm -> fused q/k/v projection -> per-head RMSNorm on q and k ->
NeoX rotary (theta) -> KV append through the reference KV quantizer -> GQA
attention over the dequantized cache -> o_proj + residual -> RMSNorm ->
softmax router (+ per-expert logit bias) top-k with renormalisation
(``expert_streaming.py:439-472``) -> SwiGLU experts (``gather_qmm`` x3,
``expert_streaming.py:224-241``) -> weighted combine + residual -> ... ->
final RMSNorm -> lm_head -> argmax.
"""

import numpy as np

from . import affine, attn, kv_sym, moe
from .fp import round_bf16


def rmsnorm(h, w, eps):
    h = np.asarray(h, np.float64)
    r = 1.0 / np.sqrt((h * h).mean(axis=-1, keepdims=True) + eps)
    return round_bf16((np.asarray(w, np.float64) * h * r).astype(np.float32))


def qmm(x, w, gs, bits):
    wq, s, b = w
    W = affine.dequantize_f32(wq, s, b, gs, bits).astype(np.float64)
    return np.asarray(x, np.float64) @ W.T


def rope(v, pos, theta, D):
    """NeoX half rotation of a [.., D] head at integer position ``pos``."""
    half = D // 2
    inv = theta ** (-(2.0 * np.arange(half)) / D)
    ang = pos * inv
    c, s_ = np.cos(ang), np.sin(ang)
    x1, x2 = v[..., :half], v[..., half:]
    out = np.empty_like(v)
    out[..., :half] = round_bf16((x1 * c - x2 * s_).astype(np.float32))
    out[..., half:] = round_bf16((x2 * c + x1 * s_).astype(np.float32))
    return out


def decode_step(model, cache, tokens, positions, route_override=None, route_log=None):
    """``model``: dict of numpy weights (see b200flash.decoder for names);
    ``cache``: per layer list of (K codes+scales, V codes+scales) per sequence
    as dicts {"k": [S,Hkv,D] float32 dequantized, "v": ...} that this call
    extends with the new token.  Returns (logits [B, V] float32, next tokens).

    ``route_override``: per layer the expert ids [B, k] to use instead of the
    oracle's own top-k (their scores are still the oracle's gates, renormalised
    over the given ids) -- to compare the rest of the step on the routing a
    kernel chose where two gates are within rounding of each other.
    ``route_log``: a list that receives per layer (own ids, gates [B, E]).
    """
    cfg = model["cfg"]
    H, D, Hq, Hkv = cfg["hidden"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"]
    gs, bits, eps, theta, kvb = cfg["group_size"], cfg["bits"], cfg["rms_eps"], cfg["rope_theta"], cfg["kv_bits"]
    B = len(tokens)
    wq, s, b = model["embed"]
    h = affine.dequantize(wq[tokens], s[tokens], b[tokens], gs, bits).astype(np.float64)
    layers = model["layers"]
    xn = rmsnorm(h, layers[0]["in_norm"], eps)
    for li, ly in enumerate(layers):
        qkv = round_bf16(qmm(xn, ly["wqkv"], gs, bits).astype(np.float32)).astype(np.float64)
        q_all = np.zeros((B, Hq, D))
        for bi in range(B):
            pos = int(positions[bi])
            heads = qkv[bi].reshape(Hq + 2 * Hkv, D)
            q = rope(rmsnorm(heads[:Hq], ly["q_norm"], eps).astype(np.float64), pos, theta, D)
            k = rope(rmsnorm(heads[Hq:Hq + Hkv], ly["k_norm"], eps).astype(np.float64), pos, theta, D)
            v = heads[Hq + Hkv:]
            kq = kv_sym.quantize_tensor(k.astype(np.float32), kvb, 64, "bf16")
            vq = kv_sym.quantize_tensor(v.astype(np.float32), kvb, 64, "bf16")
            kd = kv_sym.dequantize_tensor(*kq, kvb, k.shape, 64)
            vd = kv_sym.dequantize_tensor(*vq, kvb, v.shape, 64)
            c = cache[li][bi]
            c["k"] = np.concatenate([c["k"], kd[None]], axis=0)
            c["v"] = np.concatenate([c["v"], vd[None]], axis=0)
            q_all[bi] = q
        out, _ = attn.decode_attention(q_all, [cache[li][bi]["k"] for bi in range(B)],
                                       [cache[li][bi]["v"] for bi in range(B)])
        a = round_bf16(out).reshape(B, Hq * D).astype(np.float64)
        h = round_bf16((h + qmm(a, ly["wo"], gs, bits)).astype(np.float32)).astype(np.float64)
        xn = rmsnorm(h, ly["post_norm"], eps).astype(np.float64)
        logits_r = xn @ np.asarray(ly["wr"], np.float64).T + ly["rbias"]
        inds, scores = _route_from_logits(logits_r, cfg["top_k"], cfg["norm_topk"])
        if route_log is not None:
            z = logits_r - logits_r.max(axis=-1, keepdims=True)
            gates = np.exp(z) / np.exp(z).sum(axis=-1, keepdims=True)
            route_log.append((inds.copy(), gates))
        if route_override is not None:
            z = logits_r - logits_r.max(axis=-1, keepdims=True)
            gates = np.exp(z) / np.exp(z).sum(axis=-1, keepdims=True)
            inds = np.asarray(route_override[li], np.int64)
            scores = np.take_along_axis(gates, inds, axis=-1)
            if cfg["norm_topk"]:
                scores = scores / scores.sum(axis=-1, keepdims=True)
        E = len(ly["gate"][0])
        y = np.zeros((B, H))
        # each routed expert dequantized once, applied to all of its tokens
        for e in np.unique(inds):
            bi, j = np.nonzero(inds == e)
            g = qmm(xn[bi], tuple(t[e] for t in ly["gate"]), gs, bits)
            u = qmm(xn[bi], tuple(t[e] for t in ly["up"]), gs, bits)
            hh = round_bf16((moe.silu(g) * u).astype(np.float32)).astype(np.float64)
            yk = round_bf16(qmm(hh, tuple(t[e] for t in ly["down"]), gs, bits).astype(np.float32))
            for r in range(len(bi)):
                y[bi[r]] += scores[bi[r], j[r]] * yk[r]
        assert E > 0
        h = round_bf16((h + y).astype(np.float32)).astype(np.float64)
        nxt = layers[li + 1]["in_norm"] if li + 1 < len(layers) else model["final_norm"]
        xn = rmsnorm(h, nxt, eps).astype(np.float64)
    logits = round_bf16(qmm(xn, model["lm_head"], gs, bits).astype(np.float32))
    return logits, logits.argmax(axis=-1), inds


def _route_from_logits(logits, k, renorm):
    z = logits - logits.max(axis=-1, keepdims=True)
    g = np.exp(z)
    g /= g.sum(axis=-1, keepdims=True)
    order = np.lexsort((np.broadcast_to(np.arange(g.shape[-1]), g.shape), -g), axis=-1)
    inds = order[..., :k]
    sc = np.take_along_axis(g, inds, axis=-1)
    if renorm:
        sc = sc / sc.sum(axis=-1, keepdims=True)
    return inds, sc
