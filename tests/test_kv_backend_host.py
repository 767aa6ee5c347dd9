"""Host-side checks of the KV-cache facade (kv_cache_backend.py:326-361):
backend selection by name, keyword forwarding and the unknown-name error."""

import pytest

from b200flash.kv_cache_backend import (HybridKVCache, KVCacheBackend, PlainKVCache, QuantizedKVCache,
                                        StreamingKVCache, create_kv_cache)


@pytest.mark.parametrize("strategy,cls", [("plain", PlainKVCache), ("streaming", StreamingKVCache),
                                          ("quantized", QuantizedKVCache), ("hybrid", HybridKVCache)])
def test_create_by_name(strategy, cls):
    backend = create_kv_cache(strategy, num_layers=4, num_heads=2, head_dim=64)
    assert isinstance(backend, cls) and isinstance(backend, KVCacheBackend)


def test_unknown_strategy_raises():
    with pytest.raises(ValueError, match="Unknown KV cache strategy"):
        create_kv_cache("nonexistent")


def test_kwargs_forwarded_and_filtered():
    b = create_kv_cache("streaming", num_layers=4, num_heads=2, head_dim=64, window_size=32, key_bits=8)
    st = b.get_stats()
    assert st["window_size"] == 32 and st["strategy"] == "streaming"
    q = create_kv_cache("quantized", num_layers=2, num_heads=2, head_dim=64, key_bits=8, window_size=5)
    assert q._manager.config.key_bits == 8
    h = create_kv_cache("hybrid", num_layers=2, num_heads=2, head_dim=64, window_size=16, value_bits=2)
    assert h._stream_cache.config.window_size == 16 and h._quant_config.value_bits == 2


def test_plain_empty_and_stats():
    c = PlainKVCache(2, 4, 64)
    k, v = c.get_kv(0)
    assert tuple(k.shape) == (4, 0, 64) and tuple(v.shape) == (4, 0, 64)
    assert c.get_stats() == {"strategy": "plain", "num_layers": 2, "total_tokens": 0}
