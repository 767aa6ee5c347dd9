"""GPU parity: the grouped tcgen05 GEMM over expert-sorted rows.

Row gather into plan order -> fused SwitchGLU gate/up (output kept sorted and
column-permuted) -> down projection (output back in assignment order), the
decode/prefill MoE pipeline, against the oracle's SwiGLU experts."""

import numpy as np
import pytest
import torch

from b200flash import mx_compat
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K, bits):
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    return affine.quantize(w, 64, bits)


def _dev3(t, dev):
    wq, s, b = t
    return u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev)


def _routing(rng, T, k, E, skew):
    if skew:  # Zipf-like popularity: a few hot experts with many tokens
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        p /= p.sum()
        return np.stack([rng.choice(E, k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    return np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)


@pytest.mark.parametrize("T,k,E,H,I,tile,bits,skew", [
    (64, 8, 128, 2048, 768, 64, 4, True),     # decode step of the Qwen3-MoE shape
    (7, 2, 4, 256, 128, 16, 4, False),
    (33, 4, 16, 512, 256, 32, 4, True),
    (64, 8, 32, 512, 384, 64, 8, False),
    (200, 8, 16, 512, 256, 128, 4, True),
    (300, 2, 8, 256, 128, 256, 4, True),
])
def test_sorted_swiglu_then_down(dev, T, k, E, H, I, tile, bits, skew):
    rng = np.random.default_rng(T * 31 + E)
    g, u, d = _experts(rng, E, I, H, bits), _experts(rng, E, I, H, bits), _experts(rng, E, H, I, bits)
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    inds = _routing(rng, T, k, E, skew)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds).to(dev).reshape(-1), E, tile)
    xs = mx_compat.moe_gather_rows(to_dev(x, "bf16", dev), plan, x_row_div=k)
    h = mx_compat.sorted_qmm_tc(xs, plan, *_dev3(g, dev), 64, bits, up=_dev3(u, dev), out_sorted=True)
    y = mx_compat.sorted_qmm_tc(h, plan, *_dev3(d, dev), 64, bits, out_sorted=False)
    torch.cuda.synchronize()
    plan.check()
    _, _, yk = moe.expert_mlp(x, inds, np.ones(inds.shape), g, u, d, 64, bits)
    assert_close(to_np(y), yk.reshape(T * k, H), what=f"sorted tc T={T} E={E} tile={tile} bits={bits}")


def test_sorted_path_with_row_index_and_repeat(dev):
    """x rows through an explicit x_row_index (the expert-parallel layout), and a
    second call on the same buffers with new routing (no stale state)."""
    rng = np.random.default_rng(5)
    T, k, E, H, I = 40, 4, 16, 512, 256
    g, u, d = _experts(rng, E, I, H, 4), _experts(rng, E, I, H, 4), _experts(rng, E, H, I, 4)
    gd, ud, dd = _dev3(g, dev), _dev3(u, dev), _dev3(d, dev)
    pool = round_to(rng.standard_normal((3 * T, H)).astype(np.float32), "bf16")
    for rep in range(2):
        rows = rng.permutation(3 * T)[:T]
        inds = _routing(rng, T, k, E, True)
        xri = np.repeat(rows, k).astype(np.int32)
        plan = mx_compat.MoEPlan(torch.from_numpy(inds).to(dev).reshape(-1), E, 32)
        xs = mx_compat.moe_gather_rows(to_dev(pool, "bf16", dev), plan, x_row_index=torch.from_numpy(xri).to(dev))
        h = mx_compat.sorted_qmm_tc(xs, plan, *gd, 64, 4, up=ud, out_sorted=True)
        y = mx_compat.sorted_qmm_tc(h, plan, *dd, 64, 4, out_sorted=False)
        _, _, yk = moe.expert_mlp(pool[rows], inds, np.ones(inds.shape), g, u, d, 64, 4)
        assert_close(to_np(y), yk.reshape(T * k, H), what=f"row-index rep {rep}")
