"""GPU parity: the tcgen05/TMEM grouped GEMM (kernel c) vs the oracle."""

import numpy as np
import pytest
import torch

from b200flash import mx_compat
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _w(rng, shape, bits):
    w = round_to(rng.normal(0, 0.02, shape).astype(np.float32), "bf16")
    return affine.quantize(w, 64, bits)


def _dev3(t, dev):
    wq, s, b = t
    return u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev)


@pytest.mark.parametrize("M,N,K,bits,tile", [(16, 128, 256, 4, 16), (40, 300, 512, 4, 64), (64, 5120, 2048, 4, 64),
                                             (200, 256, 768, 4, 128), (77, 192, 1024, 8, 128),
                                             (512, 384, 2048, 4, 256)])
def test_tc_dense_matches_oracle(dev, M, N, K, bits, tile):
    rng = np.random.default_rng(M * 7 + N)
    wq, s, b = _w(rng, (N, K), bits)
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    y = mx_compat.quantized_matmul_tc(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev), 64, bits, tile=tile)
    want = affine.quantized_matmul(x, wq, s, b, True, 64, bits, out_dtype="f32")
    assert_close(to_np(y), want, what=f"tc dense M={M} N={N} K={K} bits={bits} tile={tile}")


def test_tc_dense_residual(dev):
    rng = np.random.default_rng(5)
    M, N, K = 48, 256, 512
    wq, s, b = _w(rng, (N, K), 4)
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    r = round_to(rng.standard_normal((M, N)).astype(np.float32), "bf16")
    y = mx_compat.quantized_matmul_tc(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev), 64, 4,
                                      residual=to_dev(r, "bf16", dev), tile=64)
    assert_close(to_np(y), affine.quantized_matmul(x, wq, s, b, True, 64, 4, out_dtype="f32") + r, what="residual")


@pytest.mark.parametrize("M,N,K,bits,tile,ksplit", [(64, 5120, 2048, 4, 64, 4), (64, 2048, 4096, 4, 64, 8),
                                                    (37, 300, 768, 8, 64, 3), (16, 256, 512, 4, 16, 5)])
def test_tc_dense_splitk(dev, M, N, K, bits, tile, ksplit):
    """Split-K: fp32 partials per K range, summed with the residual by a second kernel."""
    rng = np.random.default_rng(M + N + ksplit)
    wq, s, b = _w(rng, (N, K), bits)
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    r = round_to(rng.standard_normal((M, N)).astype(np.float32), "bf16")
    y = mx_compat.quantized_matmul_tc(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev), 64, bits,
                                      residual=to_dev(r, "bf16", dev), tile=tile, ksplit=ksplit)
    want = affine.quantized_matmul(x, wq, s, b, True, 64, bits, out_dtype="f32") + r
    assert_close(to_np(y), want, what=f"split-K M={M} N={N} K={K} ks={ksplit}")


@pytest.mark.parametrize("T,k,E,tile", [(64, 8, 32, 64), (512, 8, 128, 128), (7, 2, 4, 16)])
def test_tc_grouped_swiglu_and_down(dev, T, k, E, tile):
    """Qwen3-MoE expert shapes (H 2048, I 768): SwitchGLU front half then down."""
    rng = np.random.default_rng(T + E)
    H, I = 2048, 768
    g, u, d = _w(rng, (E, I, H), 4), _w(rng, (E, I, H), 4), _w(rng, (E, H, I), 4)
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    p = np.arange(1, E + 1) ** -1.1
    p /= p.sum()
    inds = np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds.reshape(-1)).to(dev), E, tile)
    h = mx_compat.gather_qmm_tc_planned(to_dev(x, "bf16", dev), plan, *_dev3(g, dev), 64, 4, x_row_div=k,
                                        up=_dev3(u, dev))
    y = mx_compat.gather_qmm_tc_planned(h, plan, *_dev3(d, dev), 64, 4)
    _, hw, yk = moe.expert_mlp(x, inds, np.ones_like(inds, np.float64), g, u, d)
    assert_close(to_np(h), hw.reshape(T * k, I), what="tc swiglu")
    # the down projection consumes the kernel's own bf16 h
    hh = to_np(h).astype(np.float64)
    want = np.zeros((T * k, H))
    for a in range(T * k):
        e = inds.reshape(-1)[a]
        want[a] = affine.dequantize_f32(d[0][e], d[1][e], d[2][e], 64, 4).astype(np.float64) @ hh[a]
    assert_close(to_np(y), want, what="tc down")
