"""GPU parity: the reference KV quantizer (byte-exact), the cache manager, and
the fused quantized-KV decode attention vs the oracle."""

import numpy as np
import pytest
import torch

from b200flash.quantized_kv_cache import (QuantizedKVCacheManager, QuantizedKVConfig, QuantizedKVEntry,
                                          decode_attention, dequantize_tensor, packed_len, quantize_tensor)
from oracle import attn, kv_sym
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np

pytestmark = pytest.mark.gpu


def test_quantize_tensor_matches_reference_vectors(golden, dev):
    z = golden("kv_sym.npz")
    n = 0
    for entry in z["__cases__"]:
        name, bits, gs, dtype = str(entry).split("|")
        bits, gs = int(bits), int(gs)
        x = to_dev(z[f"{name}/x"], dtype, dev)
        p, s, zz = quantize_tensor(x, bits, gs)
        assert np.array_equal(to_np(p), z[f"{name}/packed"]), name
        assert np.array_equal(to_np(s).view(np.uint32), z[f"{name}/scales"].view(np.uint32)), name
        assert not to_np(zz).any()
        r = dequantize_tensor(p, s, zz, bits, tuple(x.shape), gs)
        assert np.array_equal(to_np(r).view(np.uint32), z[f"{name}/restored"].view(np.uint32)), name
        n += 1
    assert n >= 100


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_512_token_chunk_config2(dev, bits):
    """The 512-token prefill chunk of 16 sequences x 8 KV heads x 128 (bf16): byte-exact."""
    rng = np.random.default_rng(bits)
    x = round_to(rng.standard_normal((16, 512, 8, 128)).astype(np.float32), "bf16")
    p, s, _ = quantize_tensor(to_dev(x, "bf16", dev), bits, 64)
    op, os_, _ = kv_sym.quantize_tensor(x, bits, 64, "bf16")
    assert np.array_equal(to_np(p), op) and np.array_equal(to_np(s), os_)


def test_empty_and_scalar_inputs(dev):
    p, s, z = quantize_tensor(torch.zeros((0,), device=dev), 4)
    assert p.shape == (0,) and s.shape == (0,)
    r = dequantize_tensor(p, s, z, 4, (0,))
    assert r.shape == (0,)


def _entry_kv(rng, S, H, D, dtype="bf16"):
    return (round_to(rng.standard_normal((S, H, D)).astype(np.float32), dtype),
            round_to(rng.standard_normal((S, H, D)).astype(np.float32), dtype))


def test_entry_calibration_and_chunks(dev):
    cfg = QuantizedKVConfig(key_bits=4, value_bits=4, group_size=64, calibration_tokens=8)
    e = QuantizedKVEntry(8, 64, cfg)
    rng = np.random.default_rng(0)
    k1, v1 = _entry_kv(rng, 4, 8, 64)
    e.append(to_dev(k1, "bf16", dev), to_dev(v1, "bf16", dev))
    assert not e._calibration_done
    k, v = e.get_keys_values()
    assert np.array_equal(to_np(k), k1)
    k2, v2 = _entry_kv(rng, 4, 8, 64)
    e.append(to_dev(k2, "bf16", dev), to_dev(v2, "bf16", dev))
    assert e._calibration_done and e._fp_keys is None
    k3, v3 = _entry_kv(rng, 5, 8, 64)
    e.append(to_dev(k3, "bf16", dev), to_dev(v3, "bf16", dev))
    assert e.length == 13 and len(e._q_keys) == 2
    k, v = e.get_keys_values()
    kc = np.concatenate([k1, k2])
    want_k = np.concatenate([kv_sym.dequantize_tensor(*kv_sym.quantize_tensor(kc, 4, 64, "bf16"), 4, kc.shape, 64),
                             kv_sym.dequantize_tensor(*kv_sym.quantize_tensor(k3, 4, 64, "bf16"), 4, k3.shape, 64)])
    assert np.array_equal(to_np(k), want_k)
    # chunk tuples equal quantize_tensor of each chunk
    pk, sk, zk, shape = e._q_keys[1]
    op, os_, _ = kv_sym.quantize_tensor(k3, 4, 64, "bf16")
    assert np.array_equal(to_np(pk), op) and np.array_equal(to_np(sk), os_) and shape == (5, 8, 64)


def test_manager_reference_behaviour(dev):
    cfg = QuantizedKVConfig(key_bits=4, value_bits=4, group_size=64, calibration_tokens=4)
    m = QuantizedKVCacheManager(cfg, num_layers=2, num_kv_heads=4, head_dim=64)
    rng = np.random.default_rng(0)
    for _ in range(10):
        for layer in range(2):
            k, v = _entry_kv(rng, 1, 4, 64)
            m.update(layer, to_dev(k, "bf16", dev), to_dev(v, "bf16", dev))
    for layer in range(2):
        k, v = m.get_kv(layer)
        assert tuple(k.shape) == (10, 4, 64)
    with pytest.raises(IndexError):
        m.update(5, k, v)
    with pytest.raises(IndexError):
        m.get_kv(-1)
    st = m.get_stats()
    assert st["total_tokens"] == 20 and st["compression_ratio"] < 1.0 and len(st["per_layer"]) == 2
    m.reset()
    assert m.entries[0].length == 0
    with pytest.raises(ValueError, match="No data"):
        m.get_kv(0)
    cfg8 = QuantizedKVConfig(key_bits=4, value_bits=4, group_size=64, calibration_tokens=0)
    m8 = QuantizedKVCacheManager(cfg8, num_layers=2, num_kv_heads=8, head_dim=128)
    for layer in range(2):
        k, v = _entry_kv(rng, 64, 8, 128)
        m8.update(layer, to_dev(k, "bf16", dev), to_dev(v, "bf16", dev))
    assert 0 < m8.get_compression_ratio() < 0.5


def _paged_case(dev, rng, B, lens, Hq, Hkv, D, bits, page):
    """Random head-major page pool holding B sequences (pages shuffled)."""
    pl = packed_len(D, bits, 64)
    ng = D // 64
    pages_per = [(L + page - 1) // page for L in lens]
    total = sum(pages_per) + 3
    perm = rng.permutation(total)
    maxp = max(pages_per)
    bt = np.zeros((B, maxp), np.int32)
    kp = np.zeros((total, Hkv, page, pl), np.uint8)
    vp = np.zeros_like(kp)
    ks = np.zeros((total, Hkv, page, ng), np.float32)
    vs = np.zeros_like(ks)
    keys, vals = [], []
    cur = 0
    for b in range(B):
        k = round_to(rng.standard_normal((lens[b], Hkv, D)).astype(np.float32), "bf16")
        v = round_to(rng.standard_normal((lens[b], Hkv, D)).astype(np.float32), "bf16")
        qk, sk, zk = kv_sym.quantize_tensor(k, bits, 64, "bf16")
        qv, sv, zv = kv_sym.quantize_tensor(v, bits, 64, "bf16")
        keys.append(kv_sym.dequantize_tensor(qk, sk, zk, bits, k.shape, 64))
        vals.append(kv_sym.dequantize_tensor(qv, sv, zv, bits, v.shape, 64))
        for j in range(pages_per[b]):
            pg = perm[cur]
            cur += 1
            bt[b, j] = pg
            t0, t1 = j * page, min(lens[b], (j + 1) * page)
            kp[pg, :, : t1 - t0] = qk[t0:t1].transpose(1, 0, 2)
            vp[pg, :, : t1 - t0] = qv[t0:t1].transpose(1, 0, 2)
            ks[pg, :, : t1 - t0] = sk[t0:t1].transpose(1, 0, 2)
            vs[pg, :, : t1 - t0] = sv[t0:t1].transpose(1, 0, 2)
    q = round_to(rng.standard_normal((B, Hq, D)).astype(np.float32), "bf16")
    T = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    return (to_dev(q, "bf16", dev), T(kp), T(ks), T(vp), T(vs), T(bt), T(np.array(lens, np.int32))), (q, keys, vals)


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("Hq,Hkv,D", [(32, 8, 128), (32, 4, 128), (24, 4, 128), (8, 8, 128), (8, 8, 64),
                                         (16, 2, 256)])
def test_decode_attention_paged(dev, bits, Hq, Hkv, D):
    rng = np.random.default_rng(bits * 1000 + Hq + D)
    lens = [1, 17, 300, 1000]
    args, (q, keys, vals) = _paged_case(dev, rng, 4, lens, Hq, Hkv, D, bits, 64)
    want, _ = attn.decode_attention(q, keys, vals)
    for n_splits in (1, 3, None):
        out = decode_attention(*args, bits=bits, page_size=64, num_kv_heads=Hkv, n_splits=n_splits)
        assert_close(to_np(out), want, what=f"attn bits={bits} splits={n_splits}")


@pytest.mark.parametrize("B,Hkv,maxlen,page", [(40, 4, 700, 64), (64, 4, 2048, 64), (9, 8, 90, 64), (3, 4, 40, 16),
                                               (24, 2, 1500, 128)])
def test_decode_attention_ragged_batch(dev, B, Hkv, maxlen, page):
    """8-bit token-row form over ragged batches: empty sequences (zero
    output), lengths off the 16-token tiles, context splits longer than some
    sequences, 16- to 128-token pages."""
    rng = np.random.default_rng(B * 7 + maxlen)
    lens = [int(v) for v in rng.integers(0, maxlen + 1, B)]
    lens[0], lens[-1] = 0, maxlen
    if B > 4:
        lens[1], lens[2] = 1, 16
    args, (q, keys, vals) = _paged_case(dev, rng, B, lens, 8 * Hkv, Hkv, 128, 8, page)
    want, _ = attn.decode_attention(q, keys, vals)
    for n_splits in (1, 2, None):
        out = to_np(decode_attention(*args, bits=8, page_size=page, num_kv_heads=Hkv, n_splits=n_splits))
        assert_close(out, want, what=f"ragged batch B={B} splits={n_splits}")
        assert np.all(out[[i for i, n in enumerate(lens) if n == 0]] == 0)


@pytest.mark.parametrize("bits", [4, 8])
def test_decode_attention_256_token_pages(dev, bits):
    """Pages too large for the shared-memory page ring (256 tokens of 8-bit
    d128 codes) go through the direct-load kernel."""
    rng = np.random.default_rng(bits + 256)
    lens = [5, 256, 700]
    args, (q, keys, vals) = _paged_case(dev, rng, 3, lens, 32, 4, 128, bits, 256)
    want, _ = attn.decode_attention(q, keys, vals)
    for n_splits in (1, 2):
        out = decode_attention(*args, bits=bits, page_size=256, num_kv_heads=4, n_splits=n_splits)
        assert_close(to_np(out), want, what=f"attn 256-token pages bits={bits} splits={n_splits}")


def test_decode_attention_config2_shape(dev):
    """Llama-3-8B heads (32q/8kv, d128), batch 16, context 8192, 8-, 4- and 2-bit KV."""
    rng = np.random.default_rng(2)
    for bits in (8, 4, 2):
        args, (q, keys, vals) = _paged_case(dev, rng, 16, [8192] * 16, 32, 8, 128, bits, 128)
        sel = [0, 7, 15]
        want, _ = attn.decode_attention(q[sel], [keys[i] for i in sel], [vals[i] for i in sel])
        out = to_np(decode_attention(*args, bits=bits, page_size=128, num_kv_heads=8))
        assert_close(out[sel], want, what=f"config2 bits={bits}")


def test_manager_fused_attention_matches_dequantized(dev):
    cfg = QuantizedKVConfig(key_bits=8, value_bits=8, group_size=64, calibration_tokens=16)
    m = QuantizedKVCacheManager(cfg, num_layers=1, num_kv_heads=4, head_dim=128)
    rng = np.random.default_rng(4)
    for S in (10, 10, 1, 1, 37):
        k, v = _entry_kv(rng, S, 4, 128)
        m.update(0, to_dev(k, "bf16", dev), to_dev(v, "bf16", dev))
    q = round_to(rng.standard_normal((16, 128)).astype(np.float32), "bf16")
    out = m.attend(0, to_dev(q, "bf16", dev))
    kk, vv = m.get_kv(0)
    want, _ = attn.decode_attention(q[None], [to_np(kk)], [to_np(vv)])
    assert_close(to_np(out), want[0], what="manager.attend")
