"""Unified KV-cache facade of ``mlx_flash_compress/kv_cache_backend.py``
(``KVCacheBackend`` at :43-73, the four backends at :81-323, the factory
``create_kv_cache`` at :326-361) over this package's CUDA caches.

Keys and values are ``[num_heads, seq_len, head_dim]`` CUDA tensors at the
interface, as in the reference.  ``QuantizedKVCache`` stores the reference KV
format (``quantized_kv_cache.QuantizedKVCacheManager``, kernels
``b2f_kv_quantize_sym`` / ``b2f_kv_dequantize_sym``) and transposes to the
manager's ``[seq, heads, dim]`` order at the boundary; ``StreamingKVCache``
evicts with the sink + window policy (``streaming_llm.StreamingLLMCache``,
kernel ``b2f_gather_tokens``); ``HybridKVCache`` runs new chunks through the
quantized store and feeds the dequantized tail to the streaming cache.
"""

from abc import ABC, abstractmethod
from typing import Any

import torch

from .quantized_kv_cache import QuantizedKVCacheManager, QuantizedKVConfig
from .streaming_llm import StreamingLLMCache, StreamingLLMConfig


class KVCacheBackend(ABC):
    """Storage strategy for per-layer K/V of shape ``[num_heads, seq_len, head_dim]``."""

    @abstractmethod
    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        """Store the new entries of ``layer_idx``; return ``(all_keys, all_values)``."""

    @abstractmethod
    def get_kv(self, layer_idx: int):
        """The current ``(keys, values)`` of ``layer_idx``."""

    @abstractmethod
    def reset(self) -> None:
        """Drop every layer's entries."""

    @abstractmethod
    def get_stats(self) -> dict:
        """Backend statistics."""


def _empty(num_heads, head_dim, like=None):
    dev = like.device if like is not None else None
    return torch.zeros(num_heads, 0, head_dim, device=dev)


class PlainKVCache(KVCacheBackend):
    """Raw K/V, concatenated along the sequence axis (no compression, no eviction)."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int):
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self._keys = [None] * num_layers
        self._values = [None] * num_layers

    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        if self._keys[layer_idx] is None:
            self._keys[layer_idx], self._values[layer_idx] = keys, values
        else:
            self._keys[layer_idx] = torch.cat([self._keys[layer_idx], keys], dim=1)
            self._values[layer_idx] = torch.cat([self._values[layer_idx], values], dim=1)
        return self._keys[layer_idx], self._values[layer_idx]

    def get_kv(self, layer_idx: int):
        if self._keys[layer_idx] is None:
            e = _empty(self.num_heads, self.head_dim)
            return e, e
        return self._keys[layer_idx], self._values[layer_idx]

    def reset(self) -> None:
        self._keys = [None] * self.num_layers
        self._values = [None] * self.num_layers

    def get_stats(self) -> dict:
        total = sum(k.shape[1] for k in self._keys if k is not None)
        return {"strategy": "plain", "num_layers": self.num_layers, "total_tokens": total}


class StreamingKVCache(KVCacheBackend):
    """Attention-sink + recent-window eviction (StreamingLLM)."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int, *, num_sink_tokens: int = 4,
                 window_size: int = 1024, eviction_batch: int = 256):
        cfg = StreamingLLMConfig(num_sink_tokens=num_sink_tokens, window_size=window_size,
                                 eviction_batch=eviction_batch)
        self._cache = StreamingLLMCache(cfg, num_layers, num_heads, head_dim)

    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        return self._cache.update(layer_idx, keys, values)

    def get_kv(self, layer_idx: int):
        return self._cache.get_kv(layer_idx)

    def reset(self) -> None:
        self._cache.reset()

    def get_stats(self) -> dict:
        stats = self._cache.get_stats()
        stats["strategy"] = "streaming"
        return stats


class QuantizedKVCache(KVCacheBackend):
    """The reference KV format behind the unified interface (2/4/8-bit, per-group absmax)."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int, *, key_bits: int = 4, value_bits: int = 4,
                 group_size: int = 64, calibration_tokens: int = 32):
        cfg = QuantizedKVConfig(key_bits=key_bits, value_bits=value_bits, group_size=group_size,
                                calibration_tokens=calibration_tokens)
        self._manager = QuantizedKVCacheManager(cfg, num_layers, num_heads, head_dim)
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim

    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        self._manager.update(layer_idx, keys.transpose(0, 1).contiguous(),
                             values.transpose(0, 1).contiguous())
        return self.get_kv(layer_idx)

    def get_kv(self, layer_idx: int):
        try:
            k, v = self._manager.get_kv(layer_idx)
        except ValueError:
            e = _empty(self.num_heads, self.head_dim)
            return e, e
        return k.transpose(0, 1), v.transpose(0, 1)

    def reset(self) -> None:
        self._manager.reset()

    def get_stats(self) -> dict:
        stats = self._manager.get_stats()
        stats["strategy"] = "quantized"
        return stats


class HybridKVCache(KVCacheBackend):
    """Quantize every incoming chunk, then bound the length with sink + window eviction.

    As in the reference, the streaming cache holds the dequantized values
    (uniform shapes for the eviction); the savings are the quantization
    round trip plus the bounded length.
    """

    def __init__(self, num_layers: int, num_heads: int, head_dim: int, *, num_sink_tokens: int = 4,
                 window_size: int = 1024, eviction_batch: int = 256, key_bits: int = 4, value_bits: int = 4,
                 group_size: int = 64, calibration_tokens: int = 32):
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self._quant_config = QuantizedKVConfig(key_bits=key_bits, value_bits=value_bits, group_size=group_size,
                                               calibration_tokens=calibration_tokens)
        self._quant_manager = QuantizedKVCacheManager(self._quant_config, num_layers, num_heads, head_dim)
        self._stream_cache = StreamingLLMCache(
            StreamingLLMConfig(num_sink_tokens=num_sink_tokens, window_size=window_size,
                               eviction_batch=eviction_batch), num_layers, num_heads, head_dim)
        self._update_count = 0

    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        if layer_idx == 0:
            self._update_count += 1
        self._quant_manager.update(layer_idx, keys.transpose(0, 1).contiguous(),
                                   values.transpose(0, 1).contiguous())
        qk, qv = self._quant_manager.get_kv(layer_idx)
        n = keys.shape[1]
        # the lossy copy of the new tokens only, back in [heads, seq, dim]
        return self._stream_cache.update(layer_idx, qk[-n:].transpose(0, 1), qv[-n:].transpose(0, 1))

    def get_kv(self, layer_idx: int):
        return self._stream_cache.get_kv(layer_idx)

    def reset(self) -> None:
        self._quant_manager.reset()
        self._stream_cache.reset()
        self._update_count = 0

    def get_stats(self) -> dict:
        return {"strategy": "hybrid", "update_count": self._update_count,
                "streaming": self._stream_cache.get_stats(), "quantization": self._quant_manager.get_stats()}


_STREAMING_KEYS = {"num_sink_tokens", "window_size", "eviction_batch"}
_QUANTIZED_KEYS = {"key_bits", "value_bits", "group_size", "calibration_tokens"}


def create_kv_cache(strategy: str = "plain", num_layers: int = 32, num_heads: int = 8, head_dim: int = 128,
                    **kwargs: Any) -> KVCacheBackend:
    """Backend by name: ``plain``, ``streaming``, ``quantized`` or ``hybrid``;
    strategy-specific keyword arguments are forwarded, the rest ignored."""
    if strategy == "plain":
        return PlainKVCache(num_layers, num_heads, head_dim)
    if strategy == "streaming":
        return StreamingKVCache(num_layers, num_heads, head_dim,
                                **{k: v for k, v in kwargs.items() if k in _STREAMING_KEYS})
    if strategy == "quantized":
        return QuantizedKVCache(num_layers, num_heads, head_dim,
                                **{k: v for k, v in kwargs.items() if k in _QUANTIZED_KEYS})
    if strategy == "hybrid":
        return HybridKVCache(num_layers, num_heads, head_dim,
                             **{k: v for k, v in kwargs.items() if k in _STREAMING_KEYS | _QUANTIZED_KEYS})
    raise ValueError(f"Unknown KV cache strategy {strategy!r}. Choose from: plain, streaming, quantized, hybrid")
