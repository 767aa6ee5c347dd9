"""GPU parity: gather_qmm (routed experts) and the fused SwitchGLU front half."""

import numpy as np
import pytest
import torch

from b200flash import mx_compat
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K, bits, gs):
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    return affine.quantize(w, gs, bits)


def _dev3(t, dev):
    wq, s, b = t
    return u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev)


@pytest.mark.parametrize("T,k,E", [(1, 8, 16), (5, 2, 4), (33, 4, 16), (64, 8, 32)])
def test_gather_qmm_switch_layout(dev, T, k, E):
    """x[T,1,1,K] with rhs_indices[T,k] -> [T,k,1,N] (expert_streaming.py:230-241 layout)."""
    rng = np.random.default_rng(T * 100 + E)
    N, K = 96, 256
    wq, s, b = _experts(rng, E, N, K, 4, 64)
    x = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    out = mx_compat.gather_qmm(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev),
                               rhs_indices=torch.from_numpy(inds).to(dev), transpose=True, group_size=64, bits=4)
    assert tuple(out.shape) == (T, k, 1, N)
    want = affine.gather_qmm(x, wq, s, b, rhs_indices=inds, group_size=64, bits=4, out_dtype="f32")
    assert_close(to_np(out), want, what="gather_qmm")


def test_gather_qmm_down_proj_layout_8bit(dev):
    """x[T,k,1,I] per assignment (the down projection) with 8-bit experts."""
    rng = np.random.default_rng(9)
    T, k, E, N, K = 7, 3, 6, 64, 768
    wq, s, b = _experts(rng, E, N, K, 8, 64)
    x = round_to(rng.standard_normal((T, k, 1, K)).astype(np.float32), "bf16")
    inds = rng.integers(0, E, (T, k)).astype(np.int32)
    out = mx_compat.gather_qmm(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev),
                               rhs_indices=torch.from_numpy(inds).to(dev), group_size=64, bits=8)
    want = affine.gather_qmm(x, wq, s, b, rhs_indices=inds, group_size=64, bits=8, out_dtype="f32")
    assert_close(to_np(out), want, what="gather_qmm 8-bit")


def test_gather_qmm_skewed_routing_and_empty_experts(dev):
    """Most assignments on one expert (several token tiles), many experts unused."""
    rng = np.random.default_rng(11)
    T, k, E, N, K = 70, 2, 64, 48, 512
    wq, s, b = _experts(rng, E, N, K, 4, 64)
    x = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    inds = np.stack([np.zeros(T, np.int32), rng.integers(1, 4, T).astype(np.int32)], axis=1)
    out = mx_compat.gather_qmm(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev),
                               rhs_indices=torch.from_numpy(inds).to(dev), group_size=64, bits=4)
    want = affine.gather_qmm(x, wq, s, b, rhs_indices=inds, group_size=64, bits=4, out_dtype="f32")
    assert_close(to_np(out), want, what="skewed gather_qmm")


def test_moe_plan_rejects_out_of_range_expert(dev):
    plan = mx_compat.MoEPlan(torch.tensor([0, 1, 9], dtype=torch.int32, device=dev), 4, 16)
    with pytest.raises(IndexError):
        plan.check()


def test_fused_switchglu_front_half(dev):
    """silu(x.Wg^T)*(x.Wu^T) in one grouped kernel, Qwen3-MoE expert shape (I=768, H=2048)."""
    rng = np.random.default_rng(5)
    T, k, E, H, I = 6, 8, 16, 2048, 768
    g = _experts(rng, E, I, H, 4, 64)
    u = _experts(rng, E, I, H, 4, 64)
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds.reshape(-1)).to(dev), E, 16)
    h = mx_compat.gather_qmv_planned(to_dev(x, "bf16", dev), plan, *_dev3(g, dev), 64, 4, x_row_div=k,
                                     up=_dev3(u, dev))
    gw = [affine.dequantize_f32(*(a[e] for a in g), 64, 4).astype(np.float64) for e in range(E)]
    uw = [affine.dequantize_f32(*(a[e] for a in u), 64, 4).astype(np.float64) for e in range(E)]
    want = np.zeros((T * k, I))
    for t in range(T):
        for j in range(k):
            e = inds[t, j]
            want[t * k + j] = moe.silu(gw[e] @ x[t]) * (uw[e] @ x[t])
    assert_close(to_np(h), want, what="fused swiglu")


@pytest.mark.parametrize("T,E,k,renorm", [(1, 128, 8, True), (64, 128, 8, True), (37, 64, 4, False)])
def test_router_topk_matches_oracle(dev, T, E, k, renorm):
    """softmax(x.Wr + bias) top-k with renormalisation (expert_streaming.py:439-472)."""
    from b200flash.moe import route_topk

    rng = np.random.default_rng(T + E)
    H = 2048
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    wr = round_to(rng.normal(0, 0.02, (E, H)).astype(np.float32), "bf16")
    bias = (-1.1 * np.log(np.arange(1, E + 1))).astype(np.float32)
    inds, scores = route_topk(to_dev(x, "bf16", dev), to_dev(wr, "bf16", dev), k,
                              torch.from_numpy(bias).to(dev), renorm)
    logits = x.astype(np.float64) @ wr.T.astype(np.float64) + bias
    g = np.exp(logits - logits.max(-1, keepdims=True))
    g /= g.sum(-1, keepdims=True)
    order = np.argsort(-g, axis=-1, kind="stable")[:, :k]
    ws = np.take_along_axis(g, order, -1)
    if renorm:
        ws = ws / ws.sum(-1, keepdims=True)
    gi = to_np(inds)
    # same expert sets (order within a token by descending gate)
    assert np.array_equal(gi, order), (gi[:2], order[:2])
    assert_close(to_np(scores), ws, rtol=1e-4, atol=1e-5, what="router scores")


def test_moe_block_matches_oracle(dev):
    """Router + SwiGLU experts + weighted combine + residual vs the oracle MoE."""
    from b200flash.moe import moe_block

    rng = np.random.default_rng(21)
    T, E, H, I, k = 9, 16, 256, 128, 4
    g = _experts(rng, E, I, H, 4, 64)
    u = _experts(rng, E, I, H, 4, 64)
    d = _experts(rng, E, H, I, 4, 64)
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
    res = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    out, inds, scores = moe_block(to_dev(x, "bf16", dev), to_dev(wr, "bf16", dev), _dev3(g, dev), _dev3(u, dev),
                                  _dev3(d, dev), k, residual=to_dev(res, "bf16", dev))
    oi, os_ = moe.route(x, wr.T, k)
    assert np.array_equal(to_np(inds), oi)
    y, _, _ = moe.expert_mlp(x, oi, os_, g, u, d)
    assert_close(to_np(out), y + res, what="moe block")


@pytest.mark.parametrize("T,E,k,tile", [(64, 128, 8, 64), (5, 16, 4, 16), (300, 64, 6, 32)])
def test_fused_route_plan_matches_separate_calls(dev, T, E, k, tile):
    """b2f_moe_route_plan (top-k + counting sort in the last block) == route_topk then moe_plan."""
    from b200flash import _capi
    from b200flash.moe import route_topk

    rng = np.random.default_rng(T + E)
    H, N = 256, 64
    x = to_dev(round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16"), "bf16", dev)
    wr = to_dev(round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16"), "bf16", dev)
    bias = torch.from_numpy(rng.normal(0, 0.5, E).astype(np.float32)).to(dev)
    inds_ref, scores_ref = route_topk(x, wr, k, bias)
    A = T * k
    nb = int(_capi.lib().b2f_moe_plan_workspace_bytes(A, E, tile))
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    gates = torch.empty(T, E, dtype=torch.float32, device=dev)
    inds = torch.empty(T, k, dtype=torch.int32, device=dev)
    scores = torch.empty(T, k, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):  # the arrival counter must reset between calls
        _capi.call("b2f_moe_route_plan", x.data_ptr(), T, H, wr.data_ptr(), bias.data_ptr(), E, k, 1,
                   gates.data_ptr(), inds.data_ptr(), scores.data_ptr(), tile, ws.data_ptr(), nb,
                   status.data_ptr(), _capi.stream_of(dev))
        torch.cuda.synchronize()
        assert torch.equal(inds, inds_ref) and torch.equal(scores, scores_ref)
        assert int(status.item()) == 0
        # the plan drives the grouped GEMM exactly like one built by b2f_moe_plan
        wq, s, b = _experts(rng, E, N, H, 4, 64)
        wd = _dev3((wq, s, b), dev)
        out = torch.empty(A, N, dtype=torch.bfloat16, device=dev)
        _capi.call("b2f_gather_qgemm_affine_tcgen05", x.data_ptr(), H, 0, k, A, E, wd[0].data_ptr(), wd[1].data_ptr(),
                   wd[2].data_ptr(), 0, 0, 0, N, H, 4, 64, tile, ws.data_ptr(), nb, out.data_ptr(), N,
                   _capi.stream_of(dev))
        want = affine.gather_qmm(to_np(x)[:, None, None, :], wq, s, b, rhs_indices=to_np(inds),
                                 group_size=64, bits=4, out_dtype="f32")
        assert_close(to_np(out).reshape(want.shape), want, what="grouped GEMM over the fused plan")
