"""GPU parity: KV eviction (kv_compression.py H2O / ScissorHands and
streaming_llm.py StreamingLLM) replayed against the reference's own recorded
outputs, the keep-list kernel at long contexts, and the head-mean attention
probabilities computed straight from packed K pages."""

import numpy as np
import pytest
import torch

from b200flash import _capi
from b200flash.kv_compression import (AttentionScoreTracker, CompressedKVCache, KVCompressionConfig,
                                      compact_pages, evict_keep_indices)
from b200flash.quantized_kv_cache import decode_attention
from b200flash.streaming_llm import StreamingLLMCache, StreamingLLMConfig
from oracle import attn, kv_evict

from helpers import to_np
from test_gpu_kv import _paged_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scoring", ["h2o", "scissorhands"])
def test_compressed_cache_replays_reference(golden, dev, scoring):
    z = golden("kv_evict.npz")
    cfg = KVCompressionConfig(budget_ratio=0.8, sink_tokens=2, recent_window=6, scoring=scoring)
    cache = CompressedKVCache(cfg, 2, 4, 8)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    for si, n in enumerate(z[f"{scoring}/steps"]):
        for li in range(2):
            key = f"{scoring}/s{si}/l{li}"
            ko, vo = cache.update(li, T(z[f"{key}/k"]), T(z[f"{key}/v"]), T(z[f"{key}/attn"]))
            assert np.array_equal(to_np(ko), z[f"{key}/k_out"]), key
            assert np.array_equal(to_np(vo), z[f"{key}/v_out"]), key
            imp = cache.tracker._importance[li]
            got = to_np(imp) if imp is not None else np.zeros(0, np.float32)
            assert np.allclose(got, z[f"{key}/imp"], rtol=1e-5, atol=1e-7), key
            if scoring == "h2o":
                assert np.allclose(to_np(cache.tracker._global_importance), z[f"{key}/gimp"], rtol=1e-5,
                                   atol=1e-7), key
    st = cache.get_stats()
    assert [st["compression_count"], st["total_evicted"]] == list(z[f"{scoring}/stats"])


def test_streaming_cache_replays_reference(golden, dev):
    z = golden("kv_evict.npz")
    cache = StreamingLLMCache(StreamingLLMConfig(num_sink_tokens=4, window_size=16), 2, 4, 8)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    for si, n in enumerate(z["stream/steps"]):
        for li in range(2):
            key = f"stream/s{si}/l{li}"
            ko, vo = cache.update(li, T(z[f"{key}/k"]), T(z[f"{key}/v"]))
            assert np.array_equal(to_np(ko), z[f"{key}/k_out"]), key
            assert np.array_equal(to_np(vo), z[f"{key}/v_out"]), key
            assert np.array_equal(to_np(cache.get_positions(li)), z[f"{key}/pos"]), key
    st = cache.get_stats()
    assert [st["eviction_count"], st["total_evicted_tokens"], st["current_length"]] == list(z["stream/stats"])


@pytest.mark.parametrize("S,sink,window,budget,kind", [
    (100000, 4, 1024, 20000, "random"), (8192, 4, 128, 1638, "ties"), (5000, 0, 0, 777, "random"),
    (300, 4, 128, 200, "uniform"), (50, 4, 128, 10, "random"), (1, 4, 16, 0, "random"), (0, 4, 16, 0, "random")])
def test_keep_indices_long_context(dev, S, sink, window, budget, kind):
    rng = np.random.default_rng(S + budget)
    if kind == "random":
        imp = rng.random(S).astype(np.float32)
    elif kind == "ties":  # few distinct values, many equal scores
        imp = rng.integers(0, 5, S).astype(np.float32) * 0.25
    else:
        imp = None
    keep, n = evict_keep_indices(None if imp is None else torch.from_numpy(imp).to(dev), S, sink, window, budget, dev)
    want = kv_evict.keep_indices(imp, S, sink, window, budget)
    assert n == len(want)
    assert np.array_equal(to_np(keep)[:n], want)


@pytest.mark.parametrize("bits,Hq,Hkv,D,splits", [(8, 32, 8, 128, 4), (4, 32, 4, 128, 1), (8, 8, 8, 64, 3),
                                                  (2, 32, 8, 128, 2),
                                                  (4, 16, 2, 256, 2)])
def test_head_mean_probs_from_packed_pages(dev, bits, Hq, Hkv, D, splits):
    rng = np.random.default_rng(bits * 100 + Hq)
    lens = [1, 63, 700, 2049]
    args, (q, keys, vals) = _paged_case(dev, rng, len(lens), lens, Hq, Hkv, D, bits, 64)
    qd, kp, ks, vp, vs, bt, sl = args
    _, means = attn.decode_attention(q, keys, vals)
    max_len = max(lens)
    out = torch.full((len(lens), max_len), -1.0, dtype=torch.float32, device=dev)
    nb = int(_capi.lib().b2f_qkv_head_mean_probs_workspace_bytes(len(lens), Hq, splits))
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    _capi.call("b2f_qkv_head_mean_probs", qd.data_ptr(), kp.data_ptr(), ks.data_ptr(), bt.data_ptr(), bt.shape[1],
               sl.data_ptr(), max_len, len(lens), Hq, Hkv, D, 64, 64, 1, bits, 64, D ** -0.5, splits,
               ws.data_ptr(), nb, out.data_ptr(), max_len, 0, 0.0, _capi.stream_of(dev))
    got = to_np(out)
    for b, L in enumerate(lens):
        assert np.allclose(got[b, :L], means[b], rtol=2e-3, atol=1e-6), b
        assert np.all(got[b, L:] == -1.0)  # nothing written past the sequence
        assert abs(got[b, :L].sum() - 1.0) < 1e-3


def test_tracker_record_decode_accumulates(dev):
    rng = np.random.default_rng(3)
    args, (q, keys, vals) = _paged_case(dev, rng, 1, [300], 8, 2, 128, 8, 64)
    qd, kp, ks, _, _, bt, _ = args
    tr = AttentionScoreTracker(2, scoring="h2o")
    for layer in (0, 1, 0):
        tr.record_decode(layer, qd[0], kp, ks, bt[0], 300, 2, 8, 64)
    _, means = attn.decode_attention(q, keys, vals)
    assert np.allclose(to_np(tr._importance[0]), 2 * means[0], rtol=2e-3, atol=1e-6)
    assert np.allclose(to_np(tr._global_importance), 3 * means[0], rtol=2e-3, atol=1e-6)


@pytest.mark.parametrize("bits,Hq,Hkv,D", [(8, 32, 8, 128), (4, 32, 4, 128), (4, 16, 2, 256), (2, 8, 8, 64)])
def test_compact_pages_then_decode(dev, bits, Hq, Hkv, D):
    """H2O keep lists applied to a paged quantized cache: every kept row's codes
    and scales move bit-exactly, and decode attention over the compacted pages
    equals the oracle's attention over the kept tokens only."""
    rng = np.random.default_rng(bits * 7 + D)
    lens = [5, 300, 1000, 64]
    page = 64
    args, (q, keys, vals) = _paged_case(dev, rng, len(lens), lens, Hq, Hkv, D, bits, page)
    qd, kp, ks, vp, vs, bt, sl = args
    _, means = attn.decode_attention(q, keys, vals)
    keeps = [kv_evict.keep_indices(means[b], L, 4, 32, max(40, L // 4)) for b, L in enumerate(lens)]
    max_keep = max(len(k) for k in keeps)
    keep = np.zeros((len(lens), max_keep), np.int32)
    for b, k in enumerate(keeps):
        keep[b, :len(k)] = k
    n_keep = np.array([len(k) for k in keeps], np.int32)
    # destination pages: a fresh pool, pages in reverse order
    total = kp.shape[0]
    btd = np.zeros(tuple(bt.shape), np.int32)
    nxt = total - 1
    for b, k in enumerate(keeps):
        for j in range((len(k) + page - 1) // page):
            btd[b, j] = nxt
            nxt -= 1
    outs = tuple(torch.zeros_like(t) for t in (kp, ks, vp, vs))
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    compact_pages(kp, ks, vp, vs, bt, T(keep), T(n_keep), T(btd), Hkv, D, bits, page, out=outs)
    torch.cuda.synchronize()
    src = [to_np(t) for t in (kp, ks, vp, vs)]
    got = [to_np(t) for t in outs]
    btn = to_np(bt)
    for b, k in enumerate(keeps):
        for i, t in enumerate(k):
            for s_arr, g_arr in zip(src, got):
                assert np.array_equal(g_arr[btd[b, i // page], :, i % page], s_arr[btn[b, t // page], :, t % page])
    out = decode_attention(qd, outs[0], outs[1], outs[2], outs[3], T(btd), T(n_keep), bits, page, Hkv)
    ref, _ = attn.decode_attention(q, [keys[b][k] for b, k in enumerate(keeps)],
                                   [vals[b][k] for b, k in enumerate(keeps)])
    assert np.allclose(to_np(out.float()), ref, rtol=1e-2, atol=2e-2)
