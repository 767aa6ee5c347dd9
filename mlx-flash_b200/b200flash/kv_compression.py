"""Drop-in for ``mlx_flash_compress/kv_compression.py`` (H2O / ScissorHands
attention-guided KV eviction) on CUDA torch tensors.

The per-token importance (mean over heads of the newest query's attention
row), its H2O accumulation / ScissorHands EMA, the keep-list selection of
``_compress_layer`` and the reindexing of keys, values and score arrays are
sm_100a kernels (``b2f_attn_row_head_mean``, ``b2f_evict_keep_indices``,
``b2f_gather_tokens``).  For the paged quantized decode path, where no
attention matrix exists, ``AttentionScoreTracker.record_decode`` computes the
same importance from the packed K pages (``b2f_qkv_head_mean_probs``).

Keys/values are ``[num_heads, seq_len, head_dim]`` as in the reference; score
arrays are float32 on the keys' device.
"""

from dataclasses import dataclass

import torch

from ._capi import call, ptr, require_cuda, stream_of

_DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


@dataclass
class KVCompressionConfig:
    budget_ratio: float = 0.2
    sink_tokens: int = 4
    recent_window: int = 128
    scoring: str = "h2o"
    quantize_evicted: bool = False


def _grow(t, n, dev):
    """Score array extended with zeros to length n (kept as is if longer)."""
    if t is None:
        return torch.zeros(n, dtype=torch.float32, device=dev)
    if t.numel() >= n:
        return t
    return torch.cat([t, torch.zeros(n - t.numel(), dtype=torch.float32, device=dev)])


def gather_tokens(x: torch.Tensor, keep: torch.Tensor, n_keep: int, axis: int = 1) -> torch.Tensor:
    """``x`` reindexed along ``axis`` by the first ``n_keep`` entries of ``keep`` (device int32)."""
    dev = require_cuda(x, keep)
    x = x.contiguous()
    outer = 1
    for d in x.shape[:axis]:
        outer *= d
    S = x.shape[axis]
    row = x.element_size()
    for d in x.shape[axis + 1:]:
        row *= d
    out = torch.empty(*x.shape[:axis], n_keep, *x.shape[axis + 1:], dtype=x.dtype, device=dev)
    call("b2f_gather_tokens", ptr(x), ptr(out), outer, S, row, ptr(keep), n_keep, stream_of(dev))
    return out


def evict_keep_indices(importance, S: int, sink: int, window: int, budget: int, device):
    """``(keep int32 [S] on device, n_keep)`` of ``_compress_layer`` (synchronises once for the count)."""
    keep = torch.empty(max(S, 1), dtype=torch.int32, device=device)
    count = torch.zeros(1, dtype=torch.int32, device=device)
    imp_len = 0 if importance is None else importance.numel()
    call("b2f_evict_keep_indices", ptr(importance), imp_len, S, sink, window, budget, ptr(keep), ptr(count),
         stream_of(device))
    return keep, int(count.item())


def compact_pages(k_pages, k_scales, v_pages, v_scales, block_table_src, keep, n_keep, block_table_dst,
                  num_kv_heads: int, head_dim: int, bits: int, page_size: int, out=None):
    """Apply per-sequence keep lists to a paged quantized cache (kernel ``b2f_kv_pages_gather``).

    ``keep``: int32 ``[B, max_keep]`` token positions (ascending, as
    ``evict_keep_indices`` returns them); ``n_keep``: int32 ``[B]``.  Kept
    token ``i`` of sequence ``b`` lands at slot ``i`` of the pages named by
    ``block_table_dst[b]``.  Head-major pages; ``out`` = optional
    ``(k_pages, k_scales, v_pages, v_scales)`` destination pools (default: the
    source pools, which then must hold ``block_table_dst``'s pages distinct
    from the source pages).  Returns the destination pools.
    """
    dev = require_cuda(k_pages, k_scales, v_pages, v_scales, block_table_src, keep, n_keep, block_table_dst)
    if out is None:
        out = (k_pages, k_scales, v_pages, v_scales)
    bts = block_table_src.to(torch.int32).contiguous()
    btd = block_table_dst.to(torch.int32).contiguous()
    if bts.shape != btd.shape:
        raise ValueError("source and destination block tables must have the same shape")
    kp = keep.to(torch.int32).contiguous()
    if kp.dim() == 1:
        kp = kp.reshape(1, -1)
    nk = n_keep.to(torch.int32).contiguous().reshape(-1)
    B = bts.shape[0]
    if kp.shape[0] != B or nk.numel() != B:
        raise ValueError("keep / n_keep must have one row per sequence")
    call("b2f_kv_pages_gather", ptr(k_pages), ptr(k_scales), ptr(v_pages), ptr(v_scales), ptr(bts), ptr(kp),
         kp.shape[1], ptr(nk), kp.shape[1], ptr(out[0]), ptr(out[1]), ptr(out[2]), ptr(out[3]), ptr(btd),
         bts.shape[1], B, num_kv_heads, head_dim, page_size, bits, stream_of(dev))
    return out


class AttentionScoreTracker:
    """Per-token importance per layer (and H2O's cross-layer total)."""

    def __init__(self, num_layers: int, max_seq_len: int = 8192, scoring: str = "h2o"):
        if scoring not in ("h2o", "scissorhands"):
            raise ValueError(f"unknown scoring {scoring!r}")
        self.num_layers = num_layers
        self.max_seq_len = max_seq_len
        self.scoring = scoring
        self._importance = [None] * num_layers
        self._global_importance = None
        self._ema_decay = 0.9

    def _targets(self, layer_idx, S, dev):
        """(layer array, mode, global array or None) ready for an update over S tokens."""
        cur = self._importance[layer_idx]
        if cur is None:
            lay, mode = torch.empty(S, dtype=torch.float32, device=dev), 0
        else:
            lay = _grow(cur, S, dev)[:S].contiguous()
            mode = 1 if self.scoring == "h2o" else 2
        glob = None
        if self.scoring == "h2o":
            glob = _grow(self._global_importance, S, dev)[:S].contiguous()
        return lay, mode, glob

    def record_attention(self, layer_idx: int, attention_weights: torch.Tensor):
        """``attention_weights`` ``[num_heads, q_len, seq_len]``: the last query row, mean over heads."""
        dev = require_cuda(attention_weights)
        w = attention_weights.contiguous()
        if w.dtype not in _DT:
            raise ValueError(f"unsupported dtype {w.dtype}")
        H, Sq, S = w.shape
        lay, mode, glob = self._targets(layer_idx, S, dev)
        row = w[:, Sq - 1, :]
        call("b2f_attn_row_head_mean", ptr(row), _DT[w.dtype], H, Sq * S, S, mode, self._ema_decay, ptr(lay),
             ptr(glob), stream_of(dev))
        self._importance[layer_idx] = lay
        if glob is not None:
            self._global_importance = glob

    def record_decode(self, layer_idx: int, q, k_pages, k_scales, block_table, seq_len: int, num_kv_heads: int,
                      bits: int, page_size: int, softmax_scale=None, group_size: int = 64,
                      token_major: bool = False, n_splits: int = None):
        """Importance of one sequence's tokens from its paged quantized K (q ``[Hq, D]`` bf16)."""
        dev = require_cuda(q, k_pages, k_scales, block_table)
        Hq, D = q.shape[-2], q.shape[-1]
        Hkv = num_kv_heads
        if softmax_scale is None:
            softmax_scale = D ** -0.5
        lay, mode, glob = self._targets(layer_idx, seq_len, dev)
        if n_splits is None:
            n_splits = max(1, min(64, seq_len // 512))
        ws = torch.empty(int(max(16, 8 * Hq * n_splits)), dtype=torch.uint8, device=dev)
        sl = torch.tensor([seq_len], dtype=torch.int32, device=dev)
        bt = block_table.to(torch.int32).reshape(1, -1).contiguous()
        head_stride, slot_stride = (1, Hkv) if token_major else (page_size, 1)
        qq = q.to(torch.bfloat16).reshape(1, Hq, D).contiguous()
        v = torch.empty(max(seq_len, 1), dtype=torch.float32, device=dev)
        st = stream_of(dev)
        call("b2f_qkv_head_mean_probs", ptr(qq), ptr(k_pages), ptr(k_scales), ptr(bt), bt.shape[1], ptr(sl),
             seq_len, 1, Hq, Hkv, D, page_size, head_stride, slot_stride, bits, group_size, float(softmax_scale),
             n_splits, ptr(ws), ws.numel(), ptr(v), seq_len, 0, 0.0, st)
        # fold the scores into the layer array (write / H2O sum / EMA) and the H2O total
        call("b2f_attn_row_head_mean", ptr(v), 2, 1, seq_len, seq_len, mode, self._ema_decay, ptr(lay), ptr(glob), st)
        self._importance[layer_idx] = lay
        if glob is not None:
            self._global_importance = glob

    def get_token_importance(self, layer_idx: int) -> torch.Tensor:
        if self.scoring == "h2o" and self._global_importance is not None:
            return self._global_importance
        if self._importance[layer_idx] is not None:
            return self._importance[layer_idx]
        return torch.zeros(1, dtype=torch.float32)

    def get_heavy_hitters(self, layer_idx: int, top_k: int) -> torch.Tensor:
        imp = self.get_token_importance(layer_idx)
        top_k = min(top_k, imp.shape[0])
        if top_k == 0:
            return torch.zeros(0, dtype=torch.int32, device=imp.device)
        return torch.argsort(-imp, stable=True)[:top_k].to(torch.int32)

    def truncate(self, keep_indices: torch.Tensor, n_keep: int = None):
        """Reindex every score array to the kept tokens (entries past an array's end are dropped)."""
        if n_keep is None:
            n_keep = keep_indices.numel()
        keep = keep_indices[:n_keep]

        def reindex(t):
            if t is None:
                return None
            valid = keep[keep < t.numel()].to(torch.int32).contiguous()
            if valid.numel() == 0:
                return None
            return gather_tokens(t.reshape(1, -1), valid, valid.numel()).reshape(-1)

        self._importance = [reindex(t) for t in self._importance]
        self._global_importance = reindex(self._global_importance)

    def reset(self):
        self._importance = [None] * self.num_layers
        self._global_importance = None


class CompressedKVCache:
    """Budgeted KV cache: sinks + recent window + the most important middle tokens."""

    def __init__(self, config: KVCompressionConfig, num_layers: int, num_heads: int, head_dim: int):
        self.config = config
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self._keys = [None] * num_layers
        self._values = [None] * num_layers
        self.tracker = AttentionScoreTracker(num_layers, scoring=config.scoring)
        self._total_tokens_seen = 0
        self._compression_count = 0
        self._total_evicted = 0

    def update(self, layer_idx: int, new_keys: torch.Tensor, new_values: torch.Tensor,
               attention_weights: torch.Tensor = None):
        require_cuda(new_keys, new_values, attention_weights)
        new_len = new_keys.shape[1]
        if layer_idx == 0:
            self._total_tokens_seen += new_len
        if self._keys[layer_idx] is None:
            self._keys[layer_idx] = new_keys.contiguous()
            self._values[layer_idx] = new_values.contiguous()
        else:
            self._keys[layer_idx] = torch.cat([self._keys[layer_idx], new_keys], dim=1)
            self._values[layer_idx] = torch.cat([self._values[layer_idx], new_values], dim=1)
        if attention_weights is not None:
            self.tracker.record_attention(layer_idx, attention_weights)
        cur_len = self._keys[layer_idx].shape[1]
        budget = self._compute_budget(cur_len)
        if cur_len > budget:
            self._compress_layer(layer_idx, budget)
        return self._keys[layer_idx], self._values[layer_idx]

    def _compute_budget(self, seq_len: int) -> int:
        return max(self.config.sink_tokens + self.config.recent_window,
                   max(1, int(seq_len * self.config.budget_ratio)))

    def _compress_layer(self, layer_idx: int, budget: int):
        k = self._keys[layer_idx]
        cur_len = k.shape[1]
        imp = self.tracker.get_token_importance(layer_idx)
        imp = imp if imp.device == k.device else None
        keep, n_keep = evict_keep_indices(imp, cur_len, self.config.sink_tokens, self.config.recent_window, budget,
                                          k.device)
        if n_keep == cur_len:
            return
        self._keys[layer_idx] = gather_tokens(k, keep, n_keep)
        self._values[layer_idx] = gather_tokens(self._values[layer_idx], keep, n_keep)
        self.tracker.truncate(keep, n_keep)
        self._compression_count += 1
        self._total_evicted += cur_len - n_keep

    def compress(self, layer_idx: int):
        if self._keys[layer_idx] is None:
            return
        cur_len = self._keys[layer_idx].shape[1]
        budget = max(self.config.sink_tokens + self.config.recent_window, int(cur_len * self.config.budget_ratio))
        self._compress_layer(layer_idx, budget)

    def get_kv(self, layer_idx: int):
        if self._keys[layer_idx] is None:
            empty = torch.zeros(self.num_heads, 0, self.head_dim)
            return empty, empty
        return self._keys[layer_idx], self._values[layer_idx]

    def get_compression_ratio(self) -> float:
        if self._total_tokens_seen == 0:
            return 1.0
        cur = self.current_length
        return float("inf") if cur == 0 else self._total_tokens_seen / cur

    @property
    def current_length(self) -> int:
        for k in self._keys:
            if k is not None:
                return k.shape[1]
        return 0

    def get_stats(self) -> dict:
        return {"current_length": self.current_length, "total_tokens_seen": self._total_tokens_seen,
                "compression_ratio": round(self.get_compression_ratio(), 2),
                "compression_count": self._compression_count, "total_evicted": self._total_evicted,
                "scoring": self.config.scoring, "budget_ratio": self.config.budget_ratio,
                "sink_tokens": self.config.sink_tokens, "recent_window": self.config.recent_window}

    def reset(self):
        self._keys = [None] * self.num_layers
        self._values = [None] * self.num_layers
        self.tracker.reset()
        self._total_tokens_seen = 0
        self._compression_count = 0
        self._total_evicted = 0


def _model_dims(model):
    num_layers = len(model.layers)
    first = model.layers[0]
    attn = getattr(first, "self_attn", None) or getattr(first, "attention", None)
    if attn is None:
        raise ValueError("Cannot find attention module on model layer. Expected .self_attn or .attention attribute.")
    num_heads = getattr(attn, "num_heads", None) or getattr(attn, "n_heads", None)
    head_dim = getattr(attn, "head_dim", None) or getattr(attn, "d_head", None)
    if num_heads is None or head_dim is None:
        raise ValueError(f"Cannot determine num_heads/head_dim from attention module. Available attributes: {dir(attn)}")
    return num_layers, num_heads, head_dim


def apply_kv_compression(model, config: KVCompressionConfig = None) -> CompressedKVCache:
    config = config or KVCompressionConfig()
    return CompressedKVCache(config, *_model_dims(model))
