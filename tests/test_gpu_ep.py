"""GPU parity: the expert-parallel MoE block (dispatch plan, local experts,
weighted partials) against the single-process oracle MoE.

W ranks are emulated on one GPU: every rank's buffers and kernels are real;
the two collectives are replaced by their definitions (the all-gather by
concatenating the send segments in rank order, the reduce-scatter by a sum
over ranks of the partials followed by each rank's slice).  The NCCL version
of the same block runs in ``test_gpu_ep_nccl.py`` when two GPUs are visible.
"""

import numpy as np
import pytest
import torch

from b200flash.distributed_experts import ExpertShard
from b200flash.ep import ExpertParallelMoE, local_expert_slice
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


def _repack(loc, m, dev):
    """b2f_mma_repack tiles of a rank's local experts: (gate, up, down)."""
    from b200flash import _capi
    from b200flash._capi import call, ptr

    out = []
    for (wq, s, b), (N, K, mat) in zip(loc, ((m.I, m.H, 2), (m.I, m.H, 2), (m.H, m.I, 1))):
        nb = int(_capi.lib().b2f_mma_packed_bytes(m.e_count, N, K, mat))
        t = torch.empty(nb, dtype=torch.uint8, device=dev)
        call("b2f_mma_repack", ptr(wq.contiguous()), ptr(s.contiguous()), ptr(b.contiguous()), m.e_count, N, K, mat,
             ptr(t), nb, _capi.stream_of(dev))
        out.append(t)
    return tuple(out)


def _emulate(dev, W, T, E, k, H, I, bits, engine, seed):
    rng = np.random.default_rng(seed)
    g = _experts(rng, E, I, H, bits)
    u = _experts(rng, E, I, H, bits)
    d = _experts(rng, E, H, I, bits)
    wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
    xs = [round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16") for _ in range(W)]
    gd, ud, dd = _dev3(g, dev), _dev3(u, dev), _dev3(d, dev)
    wr_d = to_dev(wr, "bf16", dev)
    shards = [ExpertShard(rank=r, world_size=W, total_experts=E) for r in range(W)]
    packed = engine == "mma_packed"
    ranks = [ExpertParallelMoE(sh, T, H, I, k, dev, bits=bits, engine="mma" if packed else engine) for sh in shards]
    for r, m in enumerate(ranks):
        m.x.copy_(to_dev(xs[r], "bf16", dev))
        m.route(wr_d)
    gathered = torch.cat([m.send for m in ranks])  # the all-gather
    parts = []
    for r, m in enumerate(ranks):
        if W > 1:
            m.recv.copy_(gathered)
        loc = [tuple(local_expert_slice(t, shards[r]) for t in w) for w in (gd, ud, dd)]
        m.compute(*loc, _repack(loc, m, dev) if packed else None)
        parts.append(m.part.float())
    torch.cuda.synchronize()
    total = torch.stack(parts).sum(0)  # the reduce-scatter (before slicing)
    for m in ranks:
        m.check()
    return ranks, shards, xs, wr, (g, u, d), total


@pytest.mark.parametrize("W,T,E,k,H,I,bits,engine", [
    (1, 9, 16, 4, 256, 128, 4, "gemv"),
    (2, 5, 16, 4, 256, 128, 4, "gemv"),
    (3, 7, 16, 4, 256, 128, 4, "tc"),   # 16 experts over 3 ranks: 5, 5, 6
    (4, 16, 32, 8, 512, 256, 4, "tc"),
    (2, 12, 8, 2, 256, 192, 8, "tc"),
    (8, 4, 16, 8, 256, 128, 4, "gemv"),
    (4, 16, 32, 8, 512, 256, 4, "mma"),
    (3, 7, 16, 4, 256, 128, 4, "mma"),
    (4, 16, 32, 8, 512, 256, 4, "mma_packed"),
    (2, 24, 16, 4, 256, 384, 4, "mma_packed"),
])
def test_ep_block_matches_oracle(dev, W, T, E, k, H, I, bits, engine):
    ranks, shards, xs, wr, (g, u, d), total = _emulate(dev, W, T, E, k, H, I, bits, engine, seed=W * 100 + T)
    got = to_np(total)
    for r in range(W):
        oi, osc = moe.route(xs[r], wr.T, k)
        assert np.array_equal(to_np(ranks[r].inds), oi), f"rank {r} routing"
        want, _, _ = moe.expert_mlp(xs[r], oi, osc, g, u, d, 64, bits)
        assert_close(got[r * T:(r + 1) * T], want, what=f"EP W={W} rank {r}")


def test_ep_plan_side_outputs(dev):
    """x rows, scores and local ids per gathered assignment follow the
    segment layout and the ExpertShard ownership exactly."""
    W, T, E, k, H, I = 3, 6, 16, 4, 256, 128
    ranks, shards, xs, wr, _, _ = _emulate(dev, W, T, E, k, H, I, 4, "gemv", seed=5)
    for r, m in enumerate(ranks):
        inds = np.concatenate([to_np(q.inds) for q in ranks]).reshape(-1)
        scores = np.concatenate([to_np(q.scores) for q in ranks]).reshape(-1)
        owned = shards[r].owned_experts
        mine = (inds >= owned[0]) & (inds <= owned[-1])
        want_local = np.where(mine, inds - owned[0], -1)
        assert np.array_equal(to_np(m.local), want_local)
        assert np.array_equal(to_np(m.wts), np.where(mine, scores, 0).astype(np.float32))
        a = np.arange(W * T * k)
        want_row = (a // (T * k)) * m.seg.seg_rows + (a % (T * k)) // k
        assert np.array_equal(to_np(m.x_row), want_row)
        # every owner sees exactly the assignments routed to its experts
        assert int((to_np(m.local) >= 0).sum()) == int(mine.sum())


def test_ep_plan_flags_out_of_range_ids(dev):
    W, T, E, k, H, I = 2, 3, 8, 2, 256, 128
    shards = [ExpertShard(rank=r, world_size=W, total_experts=E) for r in range(W)]
    ranks = [ExpertParallelMoE(sh, T, H, I, k, dev, engine="gemv") for sh in shards]
    rng = np.random.default_rng(3)
    g = _dev3(_experts(rng, E, I, H, 4), dev)
    u = _dev3(_experts(rng, E, I, H, 4), dev)
    dd = _dev3(_experts(rng, E, H, I, 4), dev)
    for m in ranks:
        m.x.normal_()
        m.inds.copy_(torch.tensor([[0, 5], [7, 9], [1, 2]], dtype=torch.int32))
        m.scores.fill_(0.5)
    gathered = torch.cat([m.send for m in ranks])
    m = ranks[1]
    m.recv.copy_(gathered)
    m.compute(*[tuple(local_expert_slice(t, shards[1]) for t in w) for w in (g, u, dd)])
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        m.check()
