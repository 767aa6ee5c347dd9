"""GPU: the KV-cache facade over the quantized / streaming caches (the checks
of the reference's tests/test_kv_cache_backend.py on CUDA tensors), and the
CachedSwitchLinear drop-in against the oracle."""

import numpy as np
import pytest
import torch

from b200flash.expert_streaming import CachedSwitchLinear, ResidentExpertCache
from b200flash.kv_cache_backend import HybridKVCache, PlainKVCache, QuantizedKVCache, StreamingKVCache
from oracle import affine, kv_sym
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu
H, D, L = 4, 64, 3


def _kv(dev, n, seed=0):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(H, n, D, device=dev, generator=g), torch.randn(H, n, D, device=dev, generator=g))


def test_plain_append_and_layers(dev):
    c = PlainKVCache(L, H, D)
    c.update(0, *_kv(dev, 3, 1))
    k, _ = c.update(0, *_kv(dev, 4, 2))
    assert tuple(k.shape) == (H, 7, D)
    for i in range(1, L):
        c.update(i, *_kv(dev, 3 + i, i))
    assert [c.get_kv(i)[0].shape[1] for i in range(L)] == [7, 4, 5]
    assert c.get_stats()["total_tokens"] == 16


def test_streaming_eviction_keeps_sink_and_window(dev):
    c = StreamingKVCache(L, H, D, num_sink_tokens=2, window_size=4)
    k, v = _kv(dev, 10)
    ak, av = c.update(0, k, v)
    assert ak.shape[1] == 6
    assert torch.equal(ak[:, :2], k[:, :2]) and torch.equal(ak[:, 2:], k[:, 6:])
    c.reset()
    assert c.get_kv(0)[0].shape[1] == 0


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_quantized_facade_matches_reference_format(dev, bits):
    """[heads, seq, dim] in and out; values = dequantize(quantize(x)) of the
    reference KV format on the manager's [seq, heads, dim] rows."""
    c = QuantizedKVCache(L, H, D, key_bits=bits, value_bits=bits, calibration_tokens=0)
    k, v = _kv(dev, 16)
    c.update(0, k, v)
    rk, rv = c.get_kv(0)
    assert tuple(rk.shape) == (H, 16, D) and tuple(rv.shape) == (H, 16, D)
    kt = to_np(k.transpose(0, 1).contiguous())
    q, s, z = kv_sym.quantize_tensor(kt, bits, 64)
    want = kv_sym.dequantize_tensor(q, s, z, bits, kt.shape, 64).transpose(1, 0, 2)
    assert np.array_equal(to_np(rk), want)
    diff = float((rk - k).abs().mean())
    assert 0 < diff < (1.0 if bits > 2 else 2.0)
    assert c.get_stats()["strategy"] == "quantized"
    c.reset()
    assert c.get_kv(0)[0].shape[1] == 0


def test_hybrid_quantizes_then_evicts(dev):
    c = HybridKVCache(L, H, D, num_sink_tokens=2, window_size=4, key_bits=4, value_bits=4, calibration_tokens=0)
    k, v = _kv(dev, 12)
    ak, _ = c.update(0, k, v)
    assert ak.shape[1] == 6
    keep = torch.tensor([0, 1, 8, 9, 10, 11], device=dev)
    diff = float((ak - k[:, keep]).abs().mean())
    assert 0 < diff < 1.0
    st = c.get_stats()
    assert st["strategy"] == "hybrid" and "streaming" in st and "quantization" in st


def test_cached_switch_linear_matches_oracle(dev):
    """CachedSwitchLinear over a resident shard of experts 4..11 of 16:
    global ids remapped through the lookup table, then gather_qmm."""
    rng = np.random.default_rng(0)
    E, N, K, T, k = 16, 256, 512, 5, 2
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, 64, 4)
    owned = list(range(4, 12))
    cache = ResidentExpertCache({"gate_proj": u32_to_dev(wq[owned], dev)}, {"gate_proj": to_dev(s[owned], "bf16", dev)},
                                {"gate_proj": to_dev(b[owned], "bf16", dev)}, E, expert_ids=owned)
    layer = CachedSwitchLinear(cache, "gate_proj", 64, 4)
    x = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    ids = rng.choice(owned, size=(T, k)).astype(np.int32)
    y = layer(to_dev(x, "bf16", dev), torch.from_numpy(ids).to(dev))
    assert tuple(y.shape) == (T, k, 1, N) and len(cache._indices_buffer) == 1
    want = np.zeros((T, k, 1, N))
    for t in range(T):
        for j in range(k):
            e = ids[t, j]
            want[t, j, 0] = affine.dequantize_f32(wq[e], s[e], b[e], 64, 4).astype(np.float64) @ x[t, 0, 0]
    assert_close(to_np(y), want, what="CachedSwitchLinear")
