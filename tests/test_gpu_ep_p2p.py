"""GPU parity: the expert-parallel MoE block over the library's peer-memory
exchange (b2f_ep_p2p_dispatch / _wait / _combine) against the oracle MoE.

W ranks are emulated on one GPU (``LocalPeerGroup``): every rank's region,
kernels and flag protocol are real; the kernels of one rank store into the
other emulated ranks' regions exactly as into a peer GPU's.  The phases run
so that every wait finds its flags raised (all dispatches, then every rank's
dispatch wait and experts, then every combine wait), since a wait on one
GPU must never depend on a later launch.  The two-process version runs in
``test_gpu_ep_nccl.py`` when two GPUs are visible."""

import numpy as np
import pytest
import torch

from b200flash import _capi
from b200flash.distributed_experts import ExpertShard
from b200flash.ep import ExpertParallelMoE, LocalPeerGroup, local_expert_slice
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K):
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    return affine.quantize(w, 64, 4)


def _dev3(t, dev):
    wq, s, b = t
    return u32_to_dev(wq, dev), to_dev(s, "bf16", dev), to_dev(b, "bf16", dev)


def _repack(loc, m, dev):
    from b200flash._capi import call, ptr

    out = []
    for (wq, s, b), (N, K, mat) in zip(loc, ((m.I, m.H, 2), (m.I, m.H, 2), (m.H, m.I, 1))):
        nb = int(_capi.lib().b2f_mma_packed_bytes(m.e_count, N, K, mat))
        t = torch.empty(nb, dtype=torch.uint8, device=dev)
        call("b2f_mma_repack", ptr(wq.contiguous()), ptr(s.contiguous()), ptr(b.contiguous()), m.e_count, N, K, mat,
             ptr(t), nb, _capi.stream_of(dev))
        out.append(t)
    return tuple(out)


def _mask(inds, W, E):
    per = E // W
    own = np.minimum(inds // per, W - 1)
    return np.stack([(own == d).any(-1) for d in range(W)], -1).astype(np.float32)


@pytest.mark.parametrize("W,T,E,k,H,I,engine", [
    (2, 5, 16, 4, 256, 128, "gemv"),
    (3, 7, 16, 4, 256, 128, "tc"),       # 16 experts over 3 ranks: 5, 5, 6
    (4, 16, 32, 8, 512, 256, "mma_packed"),
    (8, 8, 64, 8, 512, 256, "mma_packed"),
    (1, 9, 16, 4, 256, 128, "mma"),
])
def test_p2p_block_matches_oracle(dev, W, T, E, k, H, I, engine):
    rng = np.random.default_rng(W * 100 + T)
    g, u, d = _experts(rng, E, I, H), _experts(rng, E, I, H), _experts(rng, E, H, I)
    gd, ud, dd = _dev3(g, dev), _dev3(u, dev), _dev3(d, dev)
    wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
    wr_d = to_dev(wr, "bf16", dev)
    grp = LocalPeerGroup(W, dev)
    shards = [ExpertShard(rank=r, world_size=W, total_experts=E) for r in range(W)]
    packed = engine == "mma_packed"
    ranks = [ExpertParallelMoE(sh, T, H, I, k, dev, exchange=grp.exchange(r), engine="mma" if packed else engine)
             for r, sh in enumerate(shards)]
    locs = [[tuple(local_expert_slice(t, shards[r]) for t in w) for w in (gd, ud, dd)] for r in range(W)]
    reps = [_repack(locs[r], ranks[r], dev) if packed else None for r in range(W)]
    # two exchanges through the same regions (layers of a decode step): the
    # flags carry the exchange number, the rows of the first are overwritten
    for it in range(2):
        xs = [round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16") for _ in range(W)]
        for r, m in enumerate(ranks):
            m.x.copy_(to_dev(xs[r], "bf16", dev))
            m.route(wr_d)
        for m in ranks:
            m.dispatch_send()
        for r, m in enumerate(ranks):
            m.dispatch_wait()
            m.compute(*locs[r], reps[r])
        for m in ranks:
            m.combine_wait()
        torch.cuda.synchronize()
        for r, m in enumerate(ranks):
            m.check()
            assert int(to_np(m.ctl)[0]) == it + 1
            assert np.array_equal(to_np(m.ctl)[1:3], [0, 0])
            oi, osc = moe.route(xs[r], wr.T, k)
            assert np.array_equal(to_np(m.inds), oi), f"rank {r} routing"
            mask = _mask(oi, W, E)
            assert np.array_equal(to_np(m.mask), mask)
            got = (m.out.float().view(T, W, H) * m.mask[:, :, None]).sum(1)
            want, _, _ = moe.expert_mlp(xs[r], oi, osc, g, u, d, 64, 4)
            assert_close(to_np(got), want, what=f"p2p EP W={W} rank {r} exchange {it}")


def test_p2p_combine_rmsnorm_consumes_rows(dev):
    """The decoder's completion of the peer combine: b2f_combine_rmsnorm with
    k = W over the [T][W][H] rows weighted by the mask equals the residual
    plus the summed MoE output, normalised."""
    from b200flash._capi import call, ptr

    W, T, E, k, H, I = 4, 6, 16, 4, 256, 128
    rng = np.random.default_rng(17)
    g, u, d = _experts(rng, E, I, H), _experts(rng, E, I, H), _experts(rng, E, H, I)
    gd, ud, dd = _dev3(g, dev), _dev3(u, dev), _dev3(d, dev)
    wr_d = to_dev(round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16"), "bf16", dev)
    grp = LocalPeerGroup(W, dev)
    shards = [ExpertShard(rank=r, world_size=W, total_experts=E) for r in range(W)]
    ranks = [ExpertParallelMoE(sh, T, H, I, k, dev, exchange=grp.exchange(r), engine="gemv")
             for r, sh in enumerate(shards)]
    for m in ranks:
        m.x.normal_()
        m.route(wr_d)
    for m in ranks:
        m.dispatch_send()
    for r, m in enumerate(ranks):
        m.dispatch_wait()
        m.compute(*[tuple(local_expert_slice(t, shards[r]) for t in w) for w in (gd, ud, dd)])
    for m in ranks:
        m.combine_wait()
    m = ranks[2]
    resid = torch.randn(T, H, device=dev).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(H, device=dev)).to(torch.bfloat16)
    h_out = torch.empty_like(resid)
    xn = torch.empty_like(resid)
    call("b2f_combine_rmsnorm", ptr(resid), ptr(m.out), ptr(m.mask), T, W, ptr(nw), 1e-6, H, ptr(h_out), ptr(xn),
         _capi.stream_of(dev))
    # the decoder's form: the owner's combine + RMSNorm with the combine wait
    # folded in gives the same bits
    h2, xn2 = torch.empty_like(resid), torch.empty_like(resid)
    m.combine_rmsnorm(resid, nw, 1e-6, h2, xn2)
    torch.cuda.synchronize()
    m.check()
    assert torch.equal(h2.view(torch.int16), h_out.view(torch.int16))
    assert torch.equal(xn2.view(torch.int16), xn.view(torch.int16))
    h = resid.float() + (m.out.float().view(T, W, H) * m.mask[:, :, None]).sum(1)
    hb = h.to(torch.bfloat16).float()
    want = nw.float() * hb * torch.rsqrt((hb * hb).mean(-1, keepdim=True) + 1e-6)
    assert_close(to_np(h_out), to_np(h), what="residual + peer rows")
    assert_close(to_np(xn), to_np(want), what="RMSNorm of the combined row")


def test_p2p_wait_times_out_without_flags(dev):
    """A wait whose flags nothing raises (only rank 0 of two dispatched)
    gives up after the wait limit and reports B2F_ERR_TIMEOUT in the call's
    status word and the device status; the context stays usable and, with
    the default limit restored, the exchange completes."""
    from b200flash._capi import call

    W, T, E, k, H, I = 2, 4, 8, 2, 256, 128
    rng = np.random.default_rng(2)
    gd, ud, dd = (_dev3(_experts(rng, E, n, kk), dev) for n, kk in ((I, H), (I, H), (H, I)))
    wr_d = to_dev(round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16"), "bf16", dev)
    grp = LocalPeerGroup(W, dev)
    shards = [ExpertShard(rank=r, world_size=W, total_experts=E) for r in range(W)]
    ranks = [ExpertParallelMoE(sh, T, H, I, k, dev, exchange=grp.exchange(r), engine="gemv")
             for r, sh in enumerate(shards)]
    for m in ranks:
        m.x.normal_()
        m.route(wr_d)
    call("b2f_set_wait_limit_ns", 50_000)
    try:
        ranks[0].dispatch_send()
        ranks[0].dispatch_wait()  # rank 1's dispatch flag is never raised
        torch.cuda.synchronize()
        assert int(ranks[0].p2p_status.item()) == _capi.B2F_ERR_TIMEOUT
        assert _capi.device_status(clear=True) == _capi.B2F_ERR_TIMEOUT
        with pytest.raises(TimeoutError):
            ranks[0].check()
        # the plan's own wait (the form the decoder uses) gives up the same way
        ranks[0].p2p_status.zero_()
        ranks[0].compute(*[tuple(local_expert_slice(t, shards[0]) for t in w) for w in (gd, ud, dd)])
        torch.cuda.synchronize()
        assert int(ranks[0].p2p_status.item()) == _capi.B2F_ERR_TIMEOUT
        assert _capi.device_status(clear=True) == _capi.B2F_ERR_TIMEOUT
    finally:
        call("b2f_set_wait_limit_ns", 0)
    # rank 1 catches up; both ranks' second waits find every flag raised
    ranks[0].p2p_status.zero_()
    ranks[1].dispatch_send()
    for r, m in enumerate(ranks):
        m.dispatch_wait()
        m.compute(*[tuple(local_expert_slice(t, shards[r]) for t in w) for w in (gd, ud, dd)])
    for m in ranks:
        m.combine_wait()
    torch.cuda.synchronize()
    for m in ranks:
        m.check()
    assert _capi.device_status() == 0
