"""The CPU oracle against the golden vectors generated from the reference's own code."""

import numpy as np
import pytest

from oracle import affine, kv_sym, mixed
from oracle.fp import round_bf16, round_f16


def _kv_cases(golden):
    z = golden("kv_sym.npz")
    for entry in z["__cases__"]:
        name, bits, gs, dtype = str(entry).split("|")
        yield z, name, int(bits), int(gs), dtype


def test_kv_oracle_matches_reference_outputs(golden):
    n = 0
    for z, name, bits, gs, dtype in _kv_cases(golden):
        x = z[f"{name}/x"]
        p, s, zr = kv_sym.quantize_tensor(x, bits, gs, dtype)
        assert np.array_equal(p, z[f"{name}/packed"]), name
        assert np.array_equal(s.view(np.uint32), z[f"{name}/scales"].view(np.uint32)), name
        assert not zr.any()
        r = kv_sym.dequantize_tensor(p, s, zr, bits, x.shape, gs)
        assert np.array_equal(r.view(np.uint32), z[f"{name}/restored"].view(np.uint32)), name
        n += 1
    assert n >= 100


def test_kv_oracle_reference_thresholds():
    """The reference's own roundtrip MSE bounds (tests/test_quantized_kv_cache.py:46-119)."""
    rng = np.random.default_rng(42)
    x = rng.standard_normal(128).astype(np.float32)
    for bits, bound in ((4, 0.02), (8, 0.001), (2, 0.6)):
        p, s, z = kv_sym.quantize_tensor(x, bits, 64)
        r = kv_sym.dequantize_tensor(p, s, z, bits, x.shape, 64)
        assert float(np.mean((x - r) ** 2)) < bound
    zz = np.zeros(64, np.float32)
    p, s, z = kv_sym.quantize_tensor(zz, 4, 64)
    assert not kv_sym.dequantize_tensor(p, s, z, 4, zz.shape, 64).any()


def test_kv_oracle_sizes_and_errors():
    for bits, n in ((4, 64), (2, 32), (8, 128)):
        p, _, _ = kv_sym.quantize_tensor(np.ones(128, np.float32), bits, 64)
        assert p.shape[-1] == n
        assert kv_sym.packed_len(128, bits, 64) == n
    with pytest.raises(ValueError, match="bits must be 2, 4, or 8"):
        kv_sym.quantize_tensor(np.ones(3, np.float32), 3)
    with pytest.raises(ValueError, match="bits must be 2, 4, or 8"):
        kv_sym.dequantize_tensor(np.ones(3), np.ones(3), np.ones(3), 5, (3,))
    p, s, z = kv_sym.quantize_tensor(np.zeros((0,), np.float32), 4)
    assert p.shape == (0,) and s.shape == (0,)


def test_mixed_precision_oracle_matches_reference(golden):
    z = golden("mixed2bit.npz")
    for i in range(3):
        rows, K, gs = (int(v) for v in z[f"c{i}/meta"])
        p, s, b = mixed.requantize_4bit_to_2bit(z[f"c{i}/wq"], z[f"c{i}/scales"], z[f"c{i}/biases"], gs)
        assert np.array_equal(p, z[f"c{i}/packed2"])
        assert np.array_equal(s.view(np.uint16), z[f"c{i}/scales2"].view(np.uint16))
        assert np.array_equal(b.view(np.uint16), z[f"c{i}/biases2"].view(np.uint16))
        d = mixed.dequantize_2bit(p, s, b, K)
        assert np.array_equal(d.view(np.uint32), z[f"c{i}/deq2"].view(np.uint32))


def test_affine_oracle_vectors(golden):
    z = golden("affine.npz")
    for bits in (2, 4, 8):
        for gs in (32, 64, 128):
            k = f"b{bits}_g{gs}"
            mq, ms, mb = affine.quantize(z[f"{k}/w"], gs, bits)  # MLX's rule is the default
            assert np.array_equal(mq, z[f"mlx/{k}/wq"])
            assert np.array_equal(ms, z[f"mlx/{k}/scales"]) and np.array_equal(mb, z[f"mlx/{k}/biases"])
            assert np.array_equal(affine.dequantize(mq, ms, mb, gs, bits), z[f"mlx/{k}/deq"])
            wq, s, b = affine.quantize(z[f"{k}/w"], gs, bits, rule="minmax")
            assert np.array_equal(wq, z[f"{k}/wq"])
            assert np.array_equal(s, z[f"{k}/scales"]) and np.array_equal(b, z[f"{k}/biases"])
            assert np.array_equal(affine.dequantize(wq, s, b, gs, bits), z[f"{k}/deq"])
            # constant group: scale 0, exact reconstruction
            assert s[3, 0] == 0 and np.all(affine.dequantize(wq, s, b, gs, bits)[3, :gs] == 0.015625)
            y = affine.quantized_matmul(z[f"{k}/x"], wq, s, b, True, gs, bits)
            assert np.array_equal(y, z[f"{k}/y"])


def _group(vals, gs=64):
    g = np.zeros((1, gs), np.float32)
    g[0, :len(vals)] = vals
    return g


def test_affine_mlx_rule_known_answers():
    """MLX's affine_quantize rule, worked by hand (4-bit, n = 15, f32 steps).

    min -1, max 0.5: |min| > |max| so the edge is -1 with a positive scale
    1.5/15 = 0.1f; q0 = rint(-1/0.1f) = -10, scale = -1/-10 = 0.1f, bias = -1.
    Codes: -1 -> 0, 0.5 -> rint(1.5/0.1f) = 15, 0 -> rint(1/0.1f) = 10.
    Stored scale bf16(0.1) = 0.10009765625."""
    wq, s, b = affine.quantize(_group([-1.0, 0.5]), 64, 4)
    assert affine.unpack(wq, 4)[0, :3].tolist() == [0, 15, 10]
    assert s[0, 0] == np.float32(0.10009765625) and b[0, 0] == -1.0
    # min -0.5, max 1: the edge is the max, the scale negative: -0.1f, bias 1
    wq, s, b = affine.quantize(_group([-0.5, 1.0]), 64, 4)
    assert affine.unpack(wq, 4)[0, :3].tolist() == [15, 0, 10]
    assert s[0, 0] == np.float32(-0.10009765625) and b[0, 0] == 1.0
    # all zero: range 0 -> scale -1e-7 (|min| > |max| is false), q0 = 0 -> bias 0
    wq, s, b = affine.quantize(_group([]), 64, 4)
    assert not wq.any() and b[0, 0] == 0 and s[0, 0] == round_bf16(np.float32(-1e-7))
    # constant 0.5: scale -1e-7, edge 0.5, q0 = rint(-5e6) -> scale 0.5/q0, bias 0.5, codes 0
    wq, s, b = affine.quantize(np.full((1, 64), 0.5, np.float32), 64, 4)
    assert not wq.any() and b[0, 0] == 0.5 and s[0, 0] < 0
    assert np.all(affine.dequantize(wq, s, b, 64, 4) == 0.5)
    # equal magnitudes: the edge is the max, scale = -(2/15 in f32 = 0.13333334);
    # 1/0.13333334 = 7.4999996 so q0 = -7, scale = 1/-7, bias 1: min -1 -> 14, 0 -> 7
    wq, s, b = affine.quantize(_group([-1.0, 1.0]), 64, 4)
    assert affine.unpack(wq, 4)[0, :3].tolist() == [14, 0, 7]
    assert s[0, 0] == round_bf16(np.float32(1) / np.float32(-7)) and b[0, 0] == 1.0
    # an exact tie in q0 rounds half to even: edge 0.75, range 0.75 + 0.5 = 1.25 -> 1.25/15
    # = 0.083333336f, 0.75 / 0.083333336f = 8.9999996 -> -9 (no tie); edge 1, min -0.875
    # range 1.875/15 = 0.125 exactly, 1/0.125 = 8 -> q0 = -8, scale = -0.125, min -> 15
    wq, s, b = affine.quantize(_group([-0.875, 1.0]), 64, 4)
    assert affine.unpack(wq, 4)[0, :3].tolist() == [15, 0, 8]
    assert s[0, 0] == -0.125 and b[0, 0] == 1.0
    # 8-bit: min -1, max 0.25: scale 1.25/255, q0 = rint(-204.0) -> bias -1 and 0 is code 204
    wq, s, b = affine.quantize(_group([-1.0, 0.25]), 64, 8)
    assert affine.unpack(wq, 8)[0, :3].tolist() == [0, 255, 204]
    with pytest.raises(ValueError, match="rule"):
        affine.quantize(_group([]), 64, 4, rule="other")


def test_affine_unpack_order_and_roundtrip():
    # element k sits at bits 4*(k%8) of word k//8 (mixed_precision.py:150-171)
    words = affine.unpack(np.array([[0x76543210, 0xFEDCBA98]], np.uint32), 4)
    assert words.tolist() == [list(range(16))]
    rng = np.random.default_rng(1)
    w = round_bf16(rng.normal(0, 0.02, (8, 128)).astype(np.float32))
    for bits in (4, 8):
        wq, s, b = affine.quantize(w, 64, bits, rule="minmax")
        err = np.abs(affine.dequantize(wq, s, b, 64, bits) - w)
        assert np.all(err <= (s.repeat(64, axis=1) * 0.5 + 1e-6) * 1.01 + np.abs(w) * 2 ** -8)
        # MLX's rule moves the grid so the edge is exact: at most one step off
        # (the far end may clip), plus the bf16 rounding of scale and bias
        wq, s, b = affine.quantize(w, 64, bits)
        err = np.abs(affine.dequantize(wq, s, b, 64, bits) - w)
        assert np.all(err <= np.abs(s.repeat(64, axis=1)) * 1.02 + np.abs(w) * 2 ** -7)


def test_round_helpers():
    assert round_bf16(np.float32(1.0 + 2 ** -8)) == 1.0  # tie -> even
    assert round_bf16(np.float32(1.0 + 3 * 2 ** -8)) == np.float32(1.0 + 2 ** -6)
    assert round_f16(np.float32(65519.0)) == 65504.0


def test_q4_0_c_restatement_against_float64():
    """The C restatement of the Q4_0 shader agrees with an order-free float64 sum."""
    from oracle import q4_0

    rng = np.random.default_rng(0)
    for M, N, gs in ((3, 64, 32), (17, 512, 32), (5, 256, 64)):
        w = rng.integers(0, 256, (M, N // 2), dtype=np.uint8)
        s = (rng.random((M, N // gs)) * 0.1).astype(np.float16)
        x = rng.standard_normal(N).astype(np.float32)
        got = q4_0.gemv(w, s, x, gs)
        want = q4_0.gemv_numpy(w, s, x, gs)
        assert np.allclose(got, want, rtol=1e-4, atol=1e-4)
    # hand case: code 9 (v=1) low nibble, code 0 (v=-8) high nibble; scale 0.5
    w = np.array([[0x09] * 16], np.uint8)
    s = np.array([[0.5]], np.float16)
    x = np.arange(32, dtype=np.float32)
    assert q4_0.gemv(w, s, x, 32)[0] == np.float32(sum(0.5 * x[0::2]) - sum(4.0 * x[1::2]))


def test_fake_quant_oracle_rules():
    from oracle import sensitivity

    w = np.array([0.7, -0.35, 0.1, 0.0], np.float32)
    out, amax = sensitivity.fake_quantize_sym(w, 4, "f32")
    assert amax == np.float32(0.7)
    scale = np.float32(0.7) / np.float32(7.0)
    assert np.array_equal(out, (np.clip(np.rint(w / scale), -8, 7) * scale).astype(np.float32))
    z, za = sensitivity.fake_quantize_sym(np.zeros(4, np.float32), 8, "bf16")
    assert za == 0 and not z.any()


def _replay_compressed(z, scoring):
    """Run the oracle's eviction over the recorded update sequence."""
    from oracle import kv_evict

    steps = z[f"{scoring}/steps"]
    L = 2
    tr = kv_evict.Tracker(L, scoring)
    keys = [None] * L
    for si, n in enumerate(steps):
        for li in range(L):
            key = f"{scoring}/s{si}/l{li}"
            k = z[f"{key}/k"]
            keys[li] = k if keys[li] is None else np.concatenate([keys[li], k], axis=1)
            tr.record(li, z[f"{key}/attn"])
            S = keys[li].shape[1]
            budget = max(2 + 6, max(1, int(S * 0.8)))
            if S > budget:
                keep = kv_evict.keep_indices(tr.importance(li), S, 2, 6, budget)
                if len(keep) != S:
                    keys[li] = keys[li][:, keep, :]
                    tr.truncate(keep)
            yield key, keys[li], tr


@pytest.mark.parametrize("scoring", ["h2o", "scissorhands"])
def test_eviction_oracle_matches_reference_goldens(golden, scoring):
    z = golden("kv_evict.npz")
    for key, keys, tr in _replay_compressed(z, scoring):
        li = int(key[-1])
        assert np.array_equal(keys, z[f"{key}/k_out"]), key
        imp = tr.imp[li] if tr.imp[li] is not None else np.zeros(0, np.float32)
        assert np.allclose(imp, z[f"{key}/imp"], rtol=1e-6, atol=1e-7), key
        if scoring == "h2o":
            assert np.allclose(tr.glob, z[f"{key}/gimp"], rtol=1e-6, atol=1e-7), key


def test_streaming_oracle_matches_reference_goldens(golden):
    from oracle import kv_evict

    z = golden("kv_evict.npz")
    keys, pos, nxt = [None, None], [None, None], [0, 0]
    for si, n in enumerate(z["stream/steps"]):
        for li in range(2):
            key = f"stream/s{si}/l{li}"
            k = z[f"{key}/k"]
            p = np.arange(nxt[li], nxt[li] + n, dtype=np.int32)
            nxt[li] += n
            keys[li] = k if keys[li] is None else np.concatenate([keys[li], k], axis=1)
            pos[li] = p if pos[li] is None else np.concatenate([pos[li], p])
            keep = kv_evict.streaming_keep(keys[li].shape[1], 4, 16)
            keys[li], pos[li] = keys[li][:, keep, :], pos[li][keep]
            assert np.array_equal(keys[li], z[f"{key}/k_out"]), key
            assert np.array_equal(pos[li], z[f"{key}/pos"]), key
