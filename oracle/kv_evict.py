"""Oracle: attention-guided and sink+window KV eviction (test infrastructure only).

Restates ``mlx_flash_compress/kv_compression.py`` (AttentionScoreTracker
:59-211, CompressedKVCache._compress_layer :293-364) and
``streaming_llm.py`` (StreamingLLMCache._evict :129-160) in NumPy:

* importance of an attention row = mean over heads of the newest query's row;
  H2O adds it to the layer's and to the cross-layer array (grown with zeros,
  cut to the row's length), ScissorHands keeps an EMA with decay 0.9;
* the keep list: sink tokens, the highest-importance middle tokens (stable
  descending order: ties go to the lower position) re-sorted by position,
  then the recent window; uniform scores when the importance array is
  shorter than the cache;
* StreamingLLM keeps ``[0, sink) + [len - window, len)``.
"""

import numpy as np


def head_mean(attn):
    """``attn`` [H, Sq, S] -> float32 [S]: mean over heads of the last query row."""
    a = np.asarray(attn, np.float32)
    return a[:, -1, :].astype(np.float64).mean(axis=0).astype(np.float32)


def keep_indices(importance, S, sink, window, budget):
    """Keep list of ``_compress_layer`` (all positions when nothing is evicted)."""
    snk, win = min(sink, S), min(window, S)
    mid0, mid1 = snk, S - win
    mid_budget = max(0, budget - (snk + win))
    if S <= budget or mid1 <= mid0 or mid_budget >= mid1 - mid0:
        return np.arange(S, dtype=np.int32)
    if importance is not None and len(importance) >= S:
        mid = np.asarray(importance, np.float32)[mid0:mid1]
    else:
        mid = np.ones(mid1 - mid0, np.float32)
    order = np.argsort(-mid, kind="stable")[:mid_budget]
    sel = np.sort(order) + mid0
    return np.concatenate([np.arange(snk), sel, np.arange(mid1, S)]).astype(np.int32)


class Tracker:
    def __init__(self, num_layers, scoring="h2o", decay=0.9):
        self.scoring = scoring
        self.decay = decay
        self.imp = [None] * num_layers
        self.glob = None

    @staticmethod
    def _grow(t, n):
        if t is None:
            return np.zeros(n, np.float32)
        return t if len(t) >= n else np.concatenate([t, np.zeros(n - len(t), np.float32)])

    def record(self, layer, attn):
        v = head_mean(attn)
        S = len(v)
        cur = self.imp[layer]
        if cur is None:
            self.imp[layer] = v
        elif self.scoring == "h2o":
            self.imp[layer] = (self._grow(cur, S)[:S] + v).astype(np.float32)
        else:
            self.imp[layer] = (np.float32(self.decay) * self._grow(cur, S)[:S]
                               + np.float32(1 - self.decay) * v).astype(np.float32)
        if self.scoring == "h2o":
            self.glob = (self._grow(self.glob, S)[:S] + v).astype(np.float32)

    def importance(self, layer):
        if self.scoring == "h2o" and self.glob is not None:
            return self.glob
        return self.imp[layer]

    def truncate(self, keep):
        def re(t):
            if t is None:
                return None
            valid = keep[keep < len(t)]
            return t[valid] if len(valid) else None

        self.imp = [re(t) for t in self.imp]
        self.glob = re(self.glob)


def streaming_keep(S, sink, window):
    if S <= sink + window:
        return np.arange(S, dtype=np.int32)
    return np.concatenate([np.arange(sink), np.arange(S - window, S)]).astype(np.int32)
