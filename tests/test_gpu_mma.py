"""GPU parity: the register-dequant warp-MMA grouped GEMM (decode-sized expert
tiles) vs the oracle, and its plan-order chaining (gate/up output consumed by
the down projection without a gather)."""

import numpy as np
import pytest
import torch

from b200flash import mx_compat
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _w(rng, shape, bits=4):
    w = round_to(rng.normal(0, 0.02, shape).astype(np.float32), "bf16")
    return affine.quantize(w, 64, bits)


def _dev3(t, dev):
    wq, s, b = t
    return u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev)


def _routing(rng, T, k, E):
    p = np.arange(1, E + 1) ** -1.1
    p /= p.sum()
    return np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)]).astype(np.int32)


@pytest.mark.parametrize("tile", [16, 32])
@pytest.mark.parametrize("T,k,E,H,I", [(64, 8, 128, 2048, 768), (64, 8, 32, 2048, 768), (7, 2, 4, 640, 384),
                                       (512, 8, 128, 2048, 768), (33, 4, 16, 1024, 512), (3, 1, 4, 256, 128)])
def test_mma_swiglu_then_down(dev, T, k, E, H, I, tile):
    """SwitchGLU front half then down projection (Qwen3-MoE expert shapes and
    ragged ones: H = 640 leaves a partial CTA and idle warps in the down GEMM;
    512 tokens put up to ~200 tokens on one expert, i.e. many slots; slots of
    1-8 tokens take the one-n-tile path, 9-16 the two-n-tile path, and with
    32-token tiles 17-32 the four-n-tile path)."""
    rng = np.random.default_rng(T * 3 + E + H)
    g, u, d = _w(rng, (E, I, H)), _w(rng, (E, I, H)), _w(rng, (E, H, I))
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    inds = _routing(rng, T, k, E)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds.reshape(-1)).to(dev), E, tile)
    h = mx_compat.gather_qmm_mma_planned(to_dev(x, "bf16", dev), plan, *_dev3(g, dev), 64, 4, x_row_div=k,
                                         up=_dev3(u, dev))
    y = mx_compat.gather_qmm_mma_planned(h, plan, *_dev3(d, dev), 64, 4, x_row_div=1)
    plan.check()
    _, hw, _ = moe.expert_mlp(x, inds, np.ones_like(inds, np.float64), g, u, d)
    assert_close(to_np(h), hw.reshape(T * k, I), what="mma swiglu")
    hh = to_np(h).astype(np.float64)
    want = np.zeros((T * k, H))
    flat = inds.reshape(-1)
    for e in np.unique(flat):
        rows = np.nonzero(flat == e)[0]
        want[rows] = hh[rows] @ affine.dequantize_f32(d[0][e], d[1][e], d[2][e], 64, 4).astype(np.float64).T
    assert_close(to_np(y), want, what="mma down")


@pytest.mark.parametrize("tile", [16, 32])
def test_mma_plan_order_chain_is_exact(dev, tile):
    """gate/up written in plan order with permuted columns equals the gathered,
    permuted natural-order output bit for bit, and the down projection reading
    it gives bit-identical rows to the natural-order chain."""
    rng = np.random.default_rng(11)
    T, k, E, H, I = 64, 8, 64, 1024, 768
    g, u, d = _w(rng, (E, I, H)), _w(rng, (E, I, H)), _w(rng, (E, H, I))
    x = to_dev(round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16"), "bf16", dev)
    inds = _routing(rng, T, k, E)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds.reshape(-1)).to(dev), E, tile)
    gu = dict(up=_dev3(u, dev))
    h_nat = mx_compat.gather_qmm_mma_planned(x, plan, *_dev3(g, dev), 64, 4, x_row_div=k, **gu)
    h_pln = mx_compat.gather_qmm_mma_planned(x, plan, *_dev3(g, dev), 64, 4, x_row_div=k, out_plan_order=True, **gu)
    gathered = mx_compat.moe_gather_rows(h_nat, plan, x_row_div=1)
    assert torch.equal(h_pln.view(torch.int16), gathered.view(torch.int16))
    y_nat = mx_compat.gather_qmm_mma_planned(h_nat, plan, *_dev3(d, dev), 64, 4, x_row_div=1)
    y_pln = mx_compat.gather_qmm_mma_planned(h_pln, plan, *_dev3(d, dev), 64, 4, x_plan_order=True)
    assert torch.equal(y_nat.view(torch.int16), y_pln.view(torch.int16))


def test_mma_tile32_equals_tile16_bitwise(dev):
    """Each (row, token) value is accumulated the same way whatever number of
    tokens shares its tile, so 32-token tiles reproduce 16-token tiles bit for
    bit (skewed routing: hot experts hold 17-64 tokens)."""
    rng = np.random.default_rng(21)
    T, k, E, H, I = 64, 8, 128, 2048, 768
    g, u, d = _w(rng, (E, I, H)), _w(rng, (E, I, H)), _w(rng, (E, H, I))
    x = to_dev(round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16"), "bf16", dev)
    inds = torch.from_numpy(_routing(rng, T, k, E).reshape(-1)).to(dev)
    outs = []
    for tile in (16, 32):
        # compared in assignment order: the order of assignments inside an
        # expert's run of the plan may differ between two plan builds
        plan = mx_compat.MoEPlan(inds, E, tile)
        h_nat = mx_compat.gather_qmm_mma_planned(x, plan, *_dev3(g, dev), 64, 4, x_row_div=k, up=_dev3(u, dev))
        h = mx_compat.gather_qmm_mma_planned(x, plan, *_dev3(g, dev), 64, 4, x_row_div=k, up=_dev3(u, dev),
                                             out_plan_order=True)
        y = mx_compat.gather_qmm_mma_planned(h, plan, *_dev3(d, dev), 64, 4, x_plan_order=True)
        plan.check()
        outs.append((h_nat, y))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_mma_single_matrix_with_row_index(dev):
    """Plain gather_qmm (no fused up) with an explicit x_row_index, vs the oracle."""
    rng = np.random.default_rng(5)
    A, E, N, K, R = 300, 24, 1000, 1280, 90
    w = _w(rng, (E, N, K))
    x = round_to(rng.standard_normal((R, K)).astype(np.float32), "bf16")
    xrow = rng.integers(0, R, A).astype(np.int32)
    eid = rng.integers(0, E, A).astype(np.int32)
    plan = mx_compat.MoEPlan(torch.from_numpy(eid).to(dev), E, 16)
    y = mx_compat.gather_qmm_mma_planned(to_dev(x, "bf16", dev), plan, *_dev3(w, dev), 64, 4,
                                         x_row_index=torch.from_numpy(xrow).to(dev))
    want = np.zeros((A, N))
    deq = [affine.dequantize_f32(w[0][e], w[1][e], w[2][e], 64, 4).astype(np.float64) for e in range(E)]
    for a in range(A):
        want[a] = deq[eid[a]] @ x[xrow[a]].astype(np.float64)
    assert_close(to_np(y), want, what="mma gather_qmm")


@pytest.mark.parametrize("M,N,K", [(64, 5120, 2048), (37, 1000, 1280), (100, 2048, 4096), (1, 256, 128)])
def test_mma_wide_tile_dense_projection(dev, M, N, K):
    """64-token tiles over a one-expert plan: mx.quantized_matmul of a decode
    batch (q/k/v and o projections); M = 100 spans two slots, M = 37 leaves
    ragged token rows, N = 1000 a partial row block."""
    rng = np.random.default_rng(M + N)
    w = _w(rng, (1, N, K))
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    plan = mx_compat.MoEPlan(torch.zeros(M, dtype=torch.int32, device=dev), 1, 64)
    y = mx_compat.gather_qmm_mma_planned(to_dev(x, "bf16", dev), plan, *_dev3(w, dev), 64, 4, x_row_div=1)
    want = x.astype(np.float64) @ affine.dequantize_f32(w[0][0], w[1][0], w[2][0], 64, 4).astype(np.float64).T
    assert_close(to_np(y), want, what=f"mma dense M={M} N={N} K={K}")


@pytest.mark.parametrize("A,E,N,K,ksplit", [(64, 1, 5120, 2048, 6), (64, 1, 2048, 4096, 11), (300, 24, 1000, 1280, 4),
                                            (5, 1, 256, 128, 3)])
@pytest.mark.parametrize("tile", [16, 64])
def test_mma_splitk_partials(dev, A, E, N, K, ksplit, tile):
    """K cut into ranges of whole 128-wide chunks: the fp32 planes sum to the
    product (a one-expert plan is the dense q/k/v or o projection of a decode
    batch); ksplit beyond the chunk count is clamped.  64-token tiles: one
    unpack of each weight serves up to 64 tokens (A = 300 spans 5 slots)."""
    rng = np.random.default_rng(A + N + ksplit)
    w = _w(rng, (E, N, K))
    x = round_to(rng.standard_normal((A, K)).astype(np.float32), "bf16")
    eid = (rng.integers(0, E, A) if E > 1 else np.zeros(A)).astype(np.int32)
    plan = mx_compat.MoEPlan(torch.from_numpy(eid).to(dev), E, tile)
    parts = mx_compat.gather_qmm_mma_partials(to_dev(x, "bf16", dev), plan, *_dev3(w, dev), 64, 4, ksplit)
    hc = K // 128
    cpk = -(-hc // min(ksplit, hc))
    assert parts.shape[0] == -(-hc // cpk)  # non-empty ranges of whole chunks
    deq = [affine.dequantize_f32(w[0][e], w[1][e], w[2][e], 64, 4).astype(np.float64) for e in range(E)]
    want = np.stack([deq[eid[a]] @ x[a].astype(np.float64) for a in range(A)])
    assert_close(to_np(parts.sum(0)), want, what=f"mma split-K A={A} E={E} N={N} K={K} ks={ksplit}")


@pytest.mark.parametrize("M,N,K", [(64, 5120, 2048), (64, 2048, 4096), (37, 1000, 1280), (16, 384, 640),
                                   (8, 256, 128), (1, 512, 256), (64, 151936 // 16, 2048)])
def test_decode_partials_stream_k(dev, M, N, K):
    """The stream-K decode GEMM (the q/k/v and o shapes of a batch-64 decode
    step, ragged token counts, a partial last row block at N = 1000, one
    chunk per row at K = 128): its planes, summed in plane order, against the
    oracle's bf16-dequantized weights (the kernel rounds q*s + b to bf16 once,
    as the tcgen05 kernels do); the plane count is the one the C ABI
    reports, and a second launch gives the same bits."""
    from b200flash import _capi
    from b200flash._capi import call, ptr

    rng = np.random.default_rng(M * 7 + N + K)
    w = _w(rng, (1, N, K))
    x = round_to(rng.standard_normal((M, K)).astype(np.float32), "bf16")
    wq, sc, bi = _dev3(w, dev)
    P = int(_capi.lib().b2f_qgemm_decode_planes(M, N, K))
    assert P >= 1
    st = _capi.stream_of(dev)
    outs = []
    for _ in range(2):
        part = torch.full((P, M, N), float("nan"), dtype=torch.float32, device=dev)
        call("b2f_qgemm_affine_decode_partials", ptr(to_dev(x, "bf16", dev)), K, M, ptr(wq[0]), ptr(sc[0]),
             ptr(bi[0]), N, K, 4, 64, ptr(part), part.numel() * 4, st)
        torch.cuda.synchronize()
        outs.append(part)
    # every plane element is written (a zero where a row block has fewer pieces)
    assert not torch.isnan(outs[0]).any()
    assert torch.equal(outs[0], outs[1])
    total = outs[0][0].clone()
    for q in range(1, P):
        total += outs[0][q]
    deq = affine.dequantize(w[0][0], w[1][0], w[2][0], 64, 4, "bf16").astype(np.float64)
    want = x.astype(np.float64) @ deq.T
    assert_close(to_np(total), want, what=f"decode GEMM M={M} N={N} K={K} P={P}")


def _two_bit(rng, E, N, K):
    """Experts quantized to 4 bits, then requantized to the 2-bit cold-expert
    format by the oracle restatement of requantize_4bit_to_2bit."""
    from oracle import mixed
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, 64, 4)
    packed, s2, b2 = zip(*(mixed.requantize_4bit_to_2bit(wq[e], s[e], b[e]) for e in range(E)))
    packed, s2, b2 = np.stack(packed), np.stack(s2), np.stack(b2)
    deq = [mixed.dequantize_2bit(packed[e], s2[e], b2[e], K).astype(np.float64) for e in range(E)]
    return packed, s2, b2, deq


@pytest.mark.parametrize("sdt", ["f16", "bf16"])
def test_mma_2bit_swiglu_and_down(dev, sdt):
    """2-bit codes (the requantized cold-expert format): SwitchGLU front half
    then down, vs float64 products of the oracle's dequantized 2-bit weights
    (bf16 scale variant: the same codes with bf16-rounded scales/biases)."""
    from oracle import mixed
    rng = np.random.default_rng(21)
    T, k, E, H, I = 24, 4, 8, 1024, 384
    gp, gs, gb, gdq = _two_bit(rng, E, I, H)
    up, us, ub, udq = _two_bit(rng, E, I, H)
    dp, ds, db, ddq = _two_bit(rng, E, H, I)
    if sdt == "bf16":
        rd = lambda a: round_to(a.astype(np.float32), "bf16")  # noqa: E731
        gs, gb, us, ub, ds, db = (rd(a) for a in (gs, gb, us, ub, ds, db))
        gdq = [mixed.dequantize_2bit(gp[e], gs[e], gb[e], H).astype(np.float64) for e in range(E)]
        udq = [mixed.dequantize_2bit(up[e], us[e], ub[e], H).astype(np.float64) for e in range(E)]
        ddq = [mixed.dequantize_2bit(dp[e], ds[e], db[e], I).astype(np.float64) for e in range(E)]
    tdt = torch.float16 if sdt == "f16" else torch.bfloat16

    def dev3(p, s, b):
        w = torch.from_numpy(np.ascontiguousarray(p)).to(dev).view(torch.int32).view(torch.uint32)
        sv = torch.from_numpy(np.asarray(s, np.float32)).to(dev).to(tdt)
        bv = torch.from_numpy(np.asarray(b, np.float32)).to(dev).to(tdt)
        return w, sv, bv

    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    inds = _routing(rng, T, k, E)
    plan = mx_compat.MoEPlan(torch.from_numpy(inds.reshape(-1)).to(dev), E, 16)
    h = mx_compat.gather_qmm_2bit_planned(to_dev(x, "bf16", dev), plan, *dev3(gp, gs, gb), x_row_div=k,
                                          up=dev3(up, us, ub))
    y = mx_compat.gather_qmm_2bit_planned(h, plan, *dev3(dp, ds, db), x_row_div=1)
    plan.check()
    xs = x.astype(np.float64)
    want_h = np.zeros((T * k, I))
    for a in range(T * k):
        e = inds.reshape(-1)[a]
        g, u = gdq[e] @ xs[a // k], udq[e] @ xs[a // k]
        want_h[a] = g / (1 + np.exp(-g)) * u
    assert_close(to_np(h), want_h, what=f"2-bit swiglu ({sdt} scales)")
    hh = to_np(h).astype(np.float64)
    want_y = np.stack([ddq[inds.reshape(-1)[a]] @ hh[a] for a in range(T * k)])
    assert_close(to_np(y), want_y, what=f"2-bit down ({sdt} scales)")


@pytest.mark.parametrize("E,N,K,T,k", [(8, 768, 2048, 64, 8), (5, 384, 640, 9, 2), (3, 256, 384, 40, 3)])
def test_packed_tiles_equal_unpacked(dev, E, N, K, T, k):
    """b2f_mma_repack (codes + in-tile scales/biases) + the bulk-copy producer:
    gate/up (SwiGLU, plan-order rows) and down outputs bit-identical to the TMA
    path over MLX-layout codes, including row blocks past N (zero-filled)."""
    from b200flash import _capi
    from b200flash._capi import call, ptr

    rng = np.random.default_rng(E * 100 + N)
    g, u = _w(rng, (E, N, K)), _w(rng, (E, N, K))
    d = _w(rng, (E, K, N))
    x = to_dev(round_to(rng.standard_normal((T, K)).astype(np.float32), "bf16"), "bf16", dev)
    inds = torch.from_numpy(np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32))
    plan = mx_compat.MoEPlan(inds.reshape(-1).to(dev), E, 16)
    G, U, D = (_dev3(t, dev) for t in (g, u, d))
    lib = _capi.lib()
    st = _capi.stream_of(dev)

    def pack(w, NN, KK, mat):
        nb = int(lib.b2f_mma_packed_bytes(E, NN, KK, mat))
        out = torch.empty(nb, dtype=torch.uint8, device=dev)
        call("b2f_mma_repack", ptr(w[0]), ptr(w[1]), ptr(w[2]), E, NN, KK, mat, ptr(out), nb, st)
        return out

    pg, pu, pd = pack(G, N, K, 2), pack(U, N, K, 2), pack(D, K, N, 1)
    A = plan.A
    h_ref = mx_compat.gather_qmm_mma_planned(x, plan, *G, 64, 4, x_row_div=k, up=U, out_plan_order=True)
    y_ref = mx_compat.gather_qmm_mma_planned(h_ref, plan, *D, 64, 4, x_plan_order=True)
    h = torch.empty(A, N, dtype=torch.bfloat16, device=dev)
    y = torch.empty(A, K, dtype=torch.bfloat16, device=dev)
    call("b2f_gather_qgemm_affine_mma_packed", ptr(x), K, 0, k, 0, A, E, ptr(pg), ptr(pu), N, K, 4, 64, 16,
         ptr(plan.workspace), plan.workspace.numel(), ptr(h), N, 1, 0, 0, 0, st)
    call("b2f_gather_qgemm_affine_mma_packed", ptr(h), N, 0, 1, 1, A, E, ptr(pd), 0, K, N, 4, 64, 16,
         ptr(plan.workspace), plan.workspace.numel(), ptr(y), K, 0, 0, 0, 0, st)
    torch.cuda.synchronize()
    # rows the plan wrote (plan order, all A assignments) compare bitwise
    assert torch.equal(h.view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    # programmatic dependent launch (gate/up lets the down GEMM start early, the
    # down GEMM waits before copying its input rows): the same bits
    h2, y2 = torch.empty_like(h), torch.empty_like(y)
    call("b2f_gather_qgemm_affine_mma_packed", ptr(x), K, 0, k, 0, A, E, ptr(pg), ptr(pu), N, K, 4, 64, 16,
         ptr(plan.workspace), plan.workspace.numel(), ptr(h2), N, 1, 0, 0, 2, st)
    call("b2f_gather_qgemm_affine_mma_packed", ptr(h2), N, 0, 1, 1, A, E, ptr(pd), 0, K, N, 4, 64, 16,
         ptr(plan.workspace), plan.workspace.numel(), ptr(y2), K, 0, 0, 0, 1, st)
    torch.cuda.synchronize()
    assert torch.equal(h2.view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(y2.view(torch.int16), y_ref.view(torch.int16))


@pytest.mark.parametrize("E,N,K,T,k", [(128, 768, 2048, 64, 8), (96, 2048, 768, 64, 8), (8, 768, 2048, 64, 8),
                                       (5, 384, 640, 9, 2)])
def test_packed_streamk_ranges(dev, E, N, K, T, k):
    """Stream-K scheduling of the packed expert GEMM (every resident CTA
    streams an equal range of (item, K chunk) units; an item cut between two
    CTAs is summed by the second to finish).  The first two shapes have more
    live items than resident CTAs, so items are cut.  Outputs equal the
    whole-item grid up to the fp32 re-association of the cut items' sums (one
    bf16 rounding step, or 2^-16 of the output rms where a sum cancels to
    about zero), are bit-identical from launch to launch,
    and the arrival counters are zero again after every launch."""
    from b200flash import _capi
    from b200flash._capi import call, ptr
    from b200flash.decoder import random_qweight

    gen = torch.Generator(device=dev)
    gen.manual_seed(E + N)
    rng = np.random.default_rng(E * 7 + K)
    G, U, D = (random_qweight(shape, 4, 64, dev, gen) for shape in ((E, N, K), (E, N, K), (E, K, N)))
    x = torch.randn(T, K, device=dev, generator=gen).to(torch.bfloat16)
    inds = torch.from_numpy(_routing(rng, T, k, E) if E > 8 else
                            np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32))
    plan = mx_compat.MoEPlan(inds.reshape(-1).to(dev), E, 16)
    lib = _capi.lib()
    st = _capi.stream_of(dev)

    def pack(w, NN, KK, mat):
        nb = int(lib.b2f_mma_packed_bytes(E, NN, KK, mat))
        out = torch.empty(nb, dtype=torch.uint8, device=dev)
        call("b2f_mma_repack", ptr(w.wq), ptr(w.scales), ptr(w.biases), E, NN, KK, mat, ptr(out), nb, st)
        return out

    pg, pu, pd = pack(G, N, K, 2), pack(U, N, K, 2), pack(D, K, N, 1)
    A = plan.A
    skb = int(lib.b2f_mma_streamk_workspace_bytes())
    assert skb > 0
    ws = torch.zeros(skb, dtype=torch.uint8, device=dev)

    def run(sk, h_in=None):
        # gate/up, then down on h_in (default: this call's own gate/up rows)
        h = torch.empty(A, N, dtype=torch.bfloat16, device=dev)
        y = torch.empty(A, K, dtype=torch.bfloat16, device=dev)
        p, n = (ptr(ws), skb) if sk else (0, 0)
        call("b2f_gather_qgemm_affine_mma_packed", ptr(x), K, 0, k, 0, A, E, ptr(pg), ptr(pu), N, K, 4, 64, 16,
             ptr(plan.workspace), plan.workspace.numel(), ptr(h), N, 1, p, n, 0, st)
        call("b2f_gather_qgemm_affine_mma_packed", ptr(h if h_in is None else h_in), N, 0, 1, 1, A, E, ptr(pd), 0,
             K, N, 4, 64, 16, ptr(plan.workspace), plan.workspace.numel(), ptr(y), K, 0, p, n, 0, st)
        torch.cuda.synchronize()
        return h, y

    # the arrival counters (one int32 per resident CTA, 256-byte padded, ahead
    # of the partials) start zero and every completed launch leaves them zero
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    counters = ws[:(sms * 3 * 4 + 255) // 256 * 256]
    assert skb == counters.numel() + sms * 3 * 2 * 4096 * 4
    h0, y0 = run(False)
    h1, y1 = run(True, h0)
    assert int(counters.count_nonzero()) == 0
    h2, y2 = run(True, h0)
    assert int(counters.count_nonzero()) == 0
    plan.check()
    assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    for got, want, what in ((h1, h0, "gate/up"), (y1, y0, "down")):
        g, w = got.float(), want.float()
        # one bf16 step, plus the re-association error of a cut item's fp32
        # sum, which is absolute (a few fp32 ulps of partial sums of the
        # output's rms size) and so dominates where the sum cancels to ~0
        floor = float(w.pow(2).mean().sqrt()) * 2.0 ** -16
        assert torch.all((g - w).abs() <= w.abs() * 2.0 ** -7 + floor), what
        assert float((got.view(torch.int16) == want.view(torch.int16)).float().mean()) > 0.98, what
