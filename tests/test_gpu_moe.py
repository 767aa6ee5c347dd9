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


def _plan_arrays(plan):
    """hdr, sorted and slots of a plan workspace, at the offsets of the
    documented layout (hdr 64 B, counts, offsets, cursor, soff, sorted,
    slots; each array 16-byte aligned)."""
    A, E = plan.A, plan.E
    up = lambda v, a: (v + a - 1) // a * a  # noqa: E731
    o = 64
    o = up(o + 4 * E, 16)
    o = up(o + 4 * (E + 1), 16)
    o = up(o + 4 * E, 16)
    o = up(o + 4 * (E + 1), 16)
    off_sorted = o
    off_slots = up(o + 4 * max(A, 1), 16)
    ws = plan.workspace.cpu().numpy()
    hdr = ws[:64].view(np.int32)
    S = int(hdr[0])
    return hdr, ws[off_sorted:off_sorted + 4 * A].view(np.int32), ws[off_slots:off_slots + 16 * S].view(np.int32).reshape(S, 4)


@pytest.mark.parametrize("A,E,tile,skew", [(512, 128, 16, 1.1), (512, 128, 32, 1.1), (4096, 64, 16, 0.5),
                                           (300, 1500, 16, 1.1), (0, 8, 16, 0.0), (7, 1, 16, 0.0)])
def test_moe_plan_slot_order(dev, A, E, tile, skew):
    """The plan's slots: every assignment in exactly one slot of its expert;
    slots holding more than tile/2 assignments come first, then the rest,
    each part in expert order, so grids over the slots start their longest
    CTAs first.  E > 1024 keeps plain expert order (global-memory counters)."""
    rng = np.random.default_rng(A + E + tile)
    p = np.arange(1, E + 1, dtype=np.float64) ** -skew
    ids = rng.choice(E, size=A, p=p / p.sum()).astype(np.int32)
    plan = mx_compat.MoEPlan(torch.from_numpy(ids).to(dev), E, tile)
    plan.check()
    hdr, srt, slots = _plan_arrays(plan)
    cnt = np.bincount(ids, minlength=E)
    assert hdr[0] == int(((cnt + tile - 1) // tile).sum())
    assert np.array_equal(np.sort(srt), np.arange(A))
    seen = np.zeros(A, np.int64)
    for e, begin, c, _ in slots:
        assert 1 <= c <= tile
        assert np.all(ids[srt[begin:begin + c]] == e)
        seen[begin:begin + c] += 1
    assert np.all(seen == 1)
    heavy = slots[:, 2] > tile // 2
    key = np.stack([slots[:, 0], slots[:, 1]], 1)
    if E <= 1024:
        nh = int(heavy.sum())
        assert heavy[:nh].all() and not heavy[nh:].any()
        parts = (key[:nh], key[nh:])
    else:
        parts = (key,)
    for part in parts:  # expert order, chunks of one expert in sorted order
        order = np.lexsort((part[:, 1], part[:, 0]))
        assert np.array_equal(order, np.arange(len(part)))


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


@pytest.mark.parametrize("engine,T,k,E,N,K,bits", [
    ("mma", 1, 8, 128, 768, 2048, 4),         # Qwen3-30B-A3B gate/up at one token
    ("mma", 32, 8, 128, 768, 2048, 4),
    ("tc_sorted", 512, 8, 16, 768, 2048, 4),  # prefill density: many tokens per expert
    ("mma", 512, 8, 16, 768, 2048, 4),
    ("tc", 40, 4, 8, 128, 576, 4),            # odd group count: per-slot tcgen05
    ("gemv", 6, 2, 8, 128, 1024, 4),
    ("mma", 9, 8, 16, 256, 7168, 4),          # DeepSeek-V3 hidden size
    ("tc_sorted", 300, 8, 8, 256, 7168, 4),
    ("tc_sorted", 70, 4, 8, 128, 2048, 8),
])
def test_gather_qmm_each_engine(dev, engine, T, k, E, N, K, bits):
    """gather_qmm through each kernel it dispatches to, Zipf-skewed routing."""
    rng = np.random.default_rng(T + E + K)
    wq, s, b = _experts(rng, E, N, K, bits, 64)
    x = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    p = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    p /= p.sum()
    inds = np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    out = mx_compat.gather_qmm(to_dev(x, "bf16", dev), *_dev3((wq, s, b), dev),
                               rhs_indices=torch.from_numpy(inds).to(dev), group_size=64, bits=bits, engine=engine)
    want = affine.gather_qmm(x, wq, s, b, rhs_indices=inds, group_size=64, bits=bits, out_dtype="f32")
    assert_close(to_np(out), want, what=f"gather_qmm engine {engine}")


@pytest.mark.parametrize("T,E,want", [(1, 128, "mma"), (32, 128, "mma"), (512, 128, "mma"), (512, 16, "tc_sorted")])
def test_gather_qmm_engine_choice(T, E, want):
    assert mx_compat.gather_qmm_engine(T * 8, E, 768, 2048, 4, 64) == want


@pytest.mark.parametrize("gating,skip,renorm", [("softmax", 3.0, True), ("sigmoid", 0.0, True),
                                                ("sigmoid", 2.0, False), ("softmax", 1.5, False)])
def test_router_gating_and_lexi_skip(dev, gating, skip, renorm):
    """Sigmoid gates and the LExI skip mask (expert_streaming.py:451-460) vs the oracle."""
    from b200flash.moe import route_topk

    rng = np.random.default_rng(int(skip * 10) + len(gating))
    T, E, H, k = 96, 64, 1024, 8
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    wr = round_to(rng.normal(0, 0.06, (E, H)).astype(np.float32), "bf16")
    bias = (-0.8 * np.log(np.arange(1, E + 1))).astype(np.float32)
    inds, scores = route_topk(to_dev(x, "bf16", dev), to_dev(wr, "bf16", dev), k, torch.from_numpy(bias).to(dev),
                              renorm, gating=gating, skip_threshold=skip)
    oi, os_ = moe.route(x, wr.T, k, renorm, bias=bias, gating=gating, skip_threshold=skip)
    assert np.array_equal(to_np(inds), oi)
    got = to_np(scores)
    if skip > 0:
        # the mask must agree wherever the decision is not within rounding of the threshold
        assert np.array_equal(got == 0, os_ == 0) or np.abs(got - os_).max() < 1e-3
        assert (os_ == 0).any(), "the threshold never fired; the case tests nothing"
    assert_close(got, os_, rtol=1e-4, atol=1e-5, what=f"router {gating} skip {skip}")


@pytest.mark.parametrize("engine", ["mma", "tc_sorted", "tc", "gemv"])
def test_switch_glu_engines(dev, engine):
    """The routed SwiGLU experts through every engine switch_glu dispatches to."""
    from b200flash.moe import switch_glu

    rng = np.random.default_rng(len(engine))
    T, E, H, I, k = 40, 8, 512, 256, 4
    g, u, d = (_experts(rng, E, n, kk, 4, 64) for n, kk in ((I, H), (I, H), (H, I)))
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    y = switch_glu(to_dev(x, "bf16", dev), torch.from_numpy(inds).to(dev), _dev3(g, dev), _dev3(u, dev),
                   _dev3(d, dev), engine=engine)
    _, _, yk = moe.expert_mlp(x, inds, np.ones(inds.shape), g, u, d)
    assert_close(to_np(y), yk, what=f"switch_glu {engine}")


@pytest.mark.parametrize("gating,skip", [("softmax", 0.0), ("softmax", 2.5), ("sigmoid", 0.0)])
def test_moe_block_shared_expert(dev, gating, skip):
    """Routed experts + LExI skip + the sigmoid-gated shared expert
    (expert_streaming.py:439-472) against the oracle, end to end."""
    from b200flash.moe import moe_block

    rng = np.random.default_rng(31 + int(skip))
    T, E, H, I, Is, k = 24, 16, 512, 256, 384, 4
    g, u, d = (_experts(rng, E, n, kk, 4, 64) for n, kk in ((I, H), (I, H), (H, I)))
    sg, su, sd = (affine.quantize(round_to(rng.normal(0, 0.02, shp).astype(np.float32), "bf16"), 64, 4)
                  for shp in ((Is, H), (Is, H), (H, Is)))
    sw = round_to(rng.normal(0, 0.05, (1, H)).astype(np.float32), "bf16")
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
    res = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    out, inds, scores = moe_block(to_dev(x, "bf16", dev), to_dev(wr, "bf16", dev), _dev3(g, dev), _dev3(u, dev),
                                  _dev3(d, dev), k, residual=to_dev(res, "bf16", dev), gating=gating,
                                  skip_threshold=skip,
                                  shared=(_dev3(sg, dev), _dev3(su, dev), _dev3(sd, dev), to_dev(sw, "bf16", dev)))
    oi, os_ = moe.route(x, wr.T, k, gating=gating, skip_threshold=skip)
    assert np.array_equal(to_np(inds), oi)
    y, _, _ = moe.expert_mlp(x, oi, os_, g, u, d)
    want = y + moe.shared_expert(x, sg, su, sd, sw) + res
    assert_close(to_np(out), want, what=f"moe block + shared ({gating}, skip {skip})")
