"""GPU parity: affine quantize / dequantize / quantized_matmul vs the oracle."""

import numpy as np
import pytest
import torch

from b200flash import mx_compat
from oracle import affine
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rule", ["mlx", "minmax"])
def test_quantize_matches_golden_bit_exact(golden, dev, rule):
    z = golden("affine.npz")
    pre = "mlx/" if rule == "mlx" else ""
    for bits in (2, 4, 8):
        for gs in (32, 64, 128):
            k = f"b{bits}_g{gs}"
            wq, s, b = mx_compat.quantize(to_dev(z[f"{k}/w"], "bf16", dev), gs, bits, rule=rule)
            assert wq.dtype == torch.uint32
            assert np.array_equal(to_np(wq), z[f"{pre}{k}/wq"]), k
            assert np.array_equal(to_np(s), z[f"{pre}{k}/scales"]), k
            assert np.array_equal(to_np(b), z[f"{pre}{k}/biases"]), k
            d = mx_compat.dequantize(wq, s, b, gs, bits)
            assert np.array_equal(to_np(d), z[f"{pre}{k}/deq"]), k
    for dt in ("f16", "f32"):
        wq, s, b = mx_compat.quantize(to_dev(z[f"{dt}/w"], dt, dev), 64, 4, rule=rule)
        assert np.array_equal(to_np(wq), z[f"{pre}{dt}/wq"]) and np.array_equal(to_np(s), z[f"{pre}{dt}/scales"])
        assert np.array_equal(to_np(mx_compat.dequantize(wq, s, b, 64, 4)), z[f"{pre}{dt}/deq"])


@pytest.mark.parametrize("bits,rule", [(4, "minmax"), (8, "minmax"), (4, "mlx"), (8, "mlx")])
def test_quantize_config1_full_size_bit_exact(dev, bits, rule):
    """W[4096, 4096] ~ N(0, 0.02) bf16, group 64: packed words, scales, biases
    bit-exact (the workload's min/max rule and MLX's edge rule)."""
    rng = np.random.default_rng(0)
    w = round_to(rng.normal(0, 0.02, (4096, 4096)).astype(np.float32), "bf16")
    wq, s, b = mx_compat.quantize(to_dev(w, "bf16", dev), 64, bits, rule=rule)
    owq, os_, ob = affine.quantize(w, 64, bits, rule=rule)
    assert np.array_equal(to_np(wq), owq)
    assert np.array_equal(to_np(s), os_) and np.array_equal(to_np(b), ob)
    d = to_np(mx_compat.dequantize(wq, s, b, 64, bits))
    assert np.array_equal(d, affine.dequantize(owq, os_, ob, 64, bits))


@pytest.mark.parametrize("rule", ["mlx", "minmax"])
def test_quantize_edge_groups(dev, rule):
    w = np.zeros((7, 128), np.float32)
    w[1] = 3.0                      # constant group
    w[2, :64] = np.linspace(-1, 1, 64)
    w[3] = round_to(np.float32(1e-30) * np.arange(128), "bf16")  # tiny range
    w[4, :64] = -np.linspace(0.1, 1, 64)  # all negative
    w[4, 64:] = np.linspace(0.1, 1, 64)  # all positive
    w[5, :2] = [-0.875, 1.0]  # exact q0 (= -8)
    w[6, :2] = [-1.0, 0.5]  # edge is the min
    w = round_to(w, "bf16")
    for bits in (2, 4, 8):
        wq, s, b = mx_compat.quantize(to_dev(w, "bf16", dev), 64, bits, rule=rule)
        owq, os_, ob = affine.quantize(w, 64, bits, rule=rule)
        assert np.array_equal(to_np(wq), owq) and np.array_equal(to_np(s), os_) and np.array_equal(to_np(b), ob)


def test_dequantize_row_gather(dev):
    rng = np.random.default_rng(3)
    w = round_to(rng.normal(0, 0.02, (64, 256)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, 64, 4)
    idx = np.array([5, 0, 63, 5, 17], np.int32)
    out = mx_compat.dequantize(u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev), 64, 4,
                               row_index=torch.from_numpy(idx).to(dev))
    assert np.array_equal(to_np(out), affine.dequantize(wq[idx], s[idx], b[idx], 64, 4))


def _qmm_case(dev, M, N, K, bits, gs, seed=0, resid=False):
    rng = np.random.default_rng(seed)
    w = round_to(rng.normal(0, 0.02, (N, K)).astype(np.float32), "bf16")
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, gs, bits)
    r = round_to(rng.standard_normal((M, N)).astype(np.float32), "bf16") if resid else None
    y = mx_compat.quantized_matmul(to_dev(x, "bf16", dev), u32_to_dev(wq, dev), to_dev(s, "bf16", dev),
                                   to_dev(b, "bf16", dev), True, gs, bits,
                                   residual=None if r is None else to_dev(r, "bf16", dev))
    want = affine.quantized_matmul(x, wq, s, b, True, gs, bits, out_dtype="f32")
    if r is not None:
        want = want + r
    assert_close(to_np(y), want, what=f"qmm M={M} N={N} K={K} bits={bits} gs={gs}")


def test_qmm_config1(dev):
    """x[8, 4096] . W[4096, 4096]^T, 4-bit g64 (rel 1e-2 / abs 2e-2 in bf16)."""
    _qmm_case(dev, 8, 4096, 4096, 4, 64)
    _qmm_case(dev, 8, 4096, 4096, 8, 64)


@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 40])
def test_qmm_token_counts(dev, M):
    _qmm_case(dev, M, 512, 2048, 4, 64, seed=M)


@pytest.mark.parametrize("bits,gs,K,N", [(4, 32, 256, 100), (4, 128, 768, 64), (8, 32, 512, 48),
                                         (8, 128, 2048, 32), (4, 64, 768, 2048), (8, 64, 64, 16)])
def test_qmm_shapes(dev, bits, gs, K, N):
    _qmm_case(dev, 5, N, K, bits, gs, seed=K + N)


def test_qmm_residual(dev):
    _qmm_case(dev, 4, 256, 1024, 4, 64, resid=True)


@pytest.mark.parametrize("M,K,bits", [(1, 7168, 4), (8, 7168, 4), (64, 7168, 8), (200, 7168, 4), (8, 14336, 4),
                                      (3, 14336, 8)])
def test_qmm_large_k_group64(dev, M, K, bits):
    """K beyond 64 groups (the DeepSeek-V3 hidden size 7168, 14336) through
    quantized_matmul's dispatch (tcgen05, split over K at decode sizes)."""
    assert mx_compat.quantized_matmul_engine(M, 256, K, bits, 64) == "tc"
    _qmm_case(dev, M, 256, K, bits, 64, seed=M + K)


@pytest.mark.parametrize("engine,M,K,gs", [("gemv", 8, 2048, 64), ("tc", 8, 2048, 64), ("tc", 130, 2048, 64),
                                           ("gemv_k", 5, 4096, 32), ("gemv_k", 9, 2304, 32)])
def test_qmm_each_engine(dev, engine, M, K, gs):
    rng = np.random.default_rng(M * 7 + K)
    N = 192
    w = round_to(rng.normal(0, 0.02, (N, K)).astype(np.float32), "bf16")
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    r = round_to(rng.standard_normal((M, N)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, gs, 4)
    y = mx_compat.quantized_matmul(to_dev(x, "bf16", dev), u32_to_dev(wq, dev), to_dev(s, "bf16", dev),
                                   to_dev(b, "bf16", dev), True, gs, 4, residual=to_dev(r, "bf16", dev),
                                   engine=engine)
    want = affine.quantized_matmul(x, wq, s, b, True, gs, 4, out_dtype="f32") + r
    assert_close(to_np(y), want, what=f"qmm engine {engine} M={M} K={K} gs={gs}")


def test_qmm_gemv_refuses_too_many_groups(dev):
    x = torch.zeros(2, 4160, dtype=torch.bfloat16, device=dev)
    wq = torch.zeros(16, 4160 // 8, dtype=torch.uint32, device=dev)
    s = torch.zeros(16, 65, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError, match="64 groups"):
        mx_compat.quantized_matmul(x, wq, s, s, True, 64, 4, engine="gemv")


@pytest.mark.parametrize("rule", ["mlx", "minmax"])
def test_quantize_exact_ties(dev, rule):
    """Groups whose codes land exactly on half-integers ((w - bias) / scale =
    k + 0.5): rounding half to even must match the oracle bit for bit."""
    g = np.zeros((4, 64), np.float32)
    g[0, :32] = np.arange(32) * 0.5  # min 0, max 15.5: ties at every odd half
    g[1, :31] = np.arange(31) * 0.5 - 7.5
    g[2, :16] = np.arange(16) + 0.5
    g[2, 16] = 0.0
    g[2, 17] = 15.0
    g[3, :64] = (np.arange(64) % 31) * 0.25 - 3.75
    w = round_to(np.tile(g, (32, 2)), "bf16")
    for bits in (2, 4, 8):
        wq, s, b = mx_compat.quantize(to_dev(w, "bf16", dev), 64, bits, rule=rule)
        owq, os_, ob = affine.quantize(w, 64, bits, rule=rule)
        assert np.array_equal(to_np(wq), owq), bits
        assert np.array_equal(to_np(s), os_) and np.array_equal(to_np(b), ob), bits
