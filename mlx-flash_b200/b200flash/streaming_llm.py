"""Drop-in for ``mlx_flash_compress/streaming_llm.py``: a fixed-size KV cache
that keeps the attention-sink tokens and a recent window (StreamingLLM), on
CUDA torch tensors.

Eviction is the keep list ``[0, sink) + [len - window, len)`` from
``b2f_evict_keep_indices`` (no importance scores: no middle tokens survive)
applied by ``b2f_gather_tokens`` to keys, values and the original position
ids.  Keys/values are ``[num_heads, seq_len, head_dim]`` as in the reference.
"""

from dataclasses import dataclass

import torch

from ._capi import require_cuda
from .kv_compression import _model_dims, evict_keep_indices, gather_tokens


@dataclass
class StreamingLLMConfig:
    num_sink_tokens: int = 4
    window_size: int = 1024
    eviction_batch: int = 256


class StreamingLLMCache:
    def __init__(self, config: StreamingLLMConfig, num_layers: int, num_heads: int, head_dim: int):
        self.config = config
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self._keys = [None] * num_layers
        self._values = [None] * num_layers
        self._positions = [None] * num_layers
        self._next_pos = [0] * num_layers
        self._total_tokens_seen = 0
        self._eviction_count = 0
        self._total_evicted_tokens = 0

    def update(self, layer_idx: int, new_keys: torch.Tensor, new_values: torch.Tensor):
        dev = require_cuda(new_keys, new_values)
        new_len = new_keys.shape[1]
        if layer_idx == 0:
            self._total_tokens_seen += new_len
        start = self._next_pos[layer_idx]
        pos = torch.arange(start, start + new_len, dtype=torch.int32, device=dev)
        self._next_pos[layer_idx] = start + new_len
        if self._keys[layer_idx] is None:
            self._keys[layer_idx] = new_keys.contiguous()
            self._values[layer_idx] = new_values.contiguous()
            self._positions[layer_idx] = pos
        else:
            self._keys[layer_idx] = torch.cat([self._keys[layer_idx], new_keys], dim=1)
            self._values[layer_idx] = torch.cat([self._values[layer_idx], new_values], dim=1)
            self._positions[layer_idx] = torch.cat([self._positions[layer_idx], pos])
        if self._keys[layer_idx].shape[1] > self.max_length:
            self._evict(layer_idx)
        return self._keys[layer_idx], self._values[layer_idx]

    def _evict(self, layer_idx: int):
        k = self._keys[layer_idx]
        cur_len = k.shape[1]
        sink, window = self.config.num_sink_tokens, self.config.window_size
        if cur_len <= sink + window:
            return
        keep, n_keep = evict_keep_indices(None, cur_len, sink, window, sink + window, k.device)
        self._keys[layer_idx] = gather_tokens(k, keep, n_keep)
        self._values[layer_idx] = gather_tokens(self._values[layer_idx], keep, n_keep)
        self._positions[layer_idx] = gather_tokens(self._positions[layer_idx].reshape(1, -1), keep,
                                                   n_keep).reshape(-1)
        self._eviction_count += 1
        self._total_evicted_tokens += cur_len - n_keep

    def get_kv(self, layer_idx: int):
        if self._keys[layer_idx] is None:
            empty = torch.zeros(self.num_heads, 0, self.head_dim)
            return empty, empty
        return self._keys[layer_idx], self._values[layer_idx]

    def get_positions(self, layer_idx: int) -> torch.Tensor:
        if self._positions[layer_idx] is None:
            return torch.zeros(0, dtype=torch.int32)
        return self._positions[layer_idx]

    @property
    def current_length(self) -> int:
        for k in self._keys:
            if k is not None:
                return k.shape[1]
        return 0

    @property
    def max_length(self) -> int:
        return self.config.num_sink_tokens + self.config.window_size

    @property
    def is_full(self) -> bool:
        return self.current_length >= self.max_length

    def get_stats(self) -> dict:
        return {"current_length": self.current_length, "max_length": self.max_length, "is_full": self.is_full,
                "num_sink_tokens": self.config.num_sink_tokens, "window_size": self.config.window_size,
                "eviction_count": self._eviction_count, "total_evicted_tokens": self._total_evicted_tokens,
                "total_tokens_seen": self._total_tokens_seen}

    def reset(self):
        self._keys = [None] * self.num_layers
        self._values = [None] * self.num_layers
        self._positions = [None] * self.num_layers
        self._next_pos = [0] * self.num_layers
        self._total_tokens_seen = 0
        self._eviction_count = 0
        self._total_evicted_tokens = 0


def apply_streaming_llm(model, config: StreamingLLMConfig = None) -> StreamingLLMCache:
    config = config or StreamingLLMConfig()
    return StreamingLLMCache(config, *_model_dims(model))
