"""GPU parity of the all-to-all expert-parallel MoE (b200flash.ep_a2a) with
W = 1..8 ranks emulated on one GPU: every rank's pack, plan, expert GEMMs,
partial sums and combine are the real kernels; the two all-to-alls are
torch copies with the same splits NCCL would use.  Compared with the
single-process oracle MoE over all tokens."""

import numpy as np
import pytest
import torch

from b200flash.distributed_experts import ExpertShard
from b200flash.ep_a2a import ExpertParallelA2A, row_pitch
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


def _experts(rng, E, N, K):
    return affine.quantize(round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16"), 64, 4)


def _slice(t, lo, hi, dev):
    return u32_to_dev(t[0][lo:hi], dev), to_dev(t[1][lo:hi], "bf16", dev), to_dev(t[2][lo:hi], "bf16", dev)


def _run(dev, W, Ts, E, H, I, k, engine, seed, skip_rank=None):
    rng = np.random.default_rng(seed)
    g, u, d = _experts(rng, E, I, H), _experts(rng, E, I, H), _experts(rng, E, H, I)
    p = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    p = p[rng.permutation(E)]
    p /= p.sum()
    xs, inds, scores = [], [], []
    for r in range(W):
        x = round_to(rng.standard_normal((Ts[r], H)).astype(np.float32), "bf16")
        pr = p.copy()
        if skip_rank is not None:  # no token routes to this rank's experts
            sh = ExpertShard(rank=skip_rank, world_size=W, total_experts=E)
            pr[sh.owned_experts] = 0
            pr /= pr.sum()
        ii = np.stack([rng.choice(E, size=k, replace=False, p=pr) for _ in range(Ts[r])]).astype(np.int32) \
            if Ts[r] else np.zeros((0, k), np.int32)
        sc = rng.uniform(0.05, 1, (Ts[r], k)).astype(np.float32)
        sc /= np.maximum(sc.sum(-1, keepdims=True), 1e-9)
        xs.append(x)
        inds.append(ii)
        scores.append(sc)
    ranks = []
    for r in range(W):
        sh = ExpertShard(rank=r, world_size=W, total_experts=E)
        ep = ExpertParallelA2A(sh, max(max(Ts), 1), H, I, k, dev, engine=engine)
        lo, hi = sh.owned_experts[0], sh.owned_experts[-1] + 1
        ranks.append((ep, _slice(g, lo, hi, dev), _slice(u, lo, hi, dev), _slice(d, lo, hi, dev)))
    dx = [to_dev(x, "bf16", dev) for x in xs]
    for r, (ep, *_w) in enumerate(ranks):
        ep.pack(dx[r], torch.from_numpy(inds[r]).to(dev), torch.from_numpy(scores[r]).to(dev))
    counts = np.stack([to_np(ep.send_counts) for ep, *_ in ranks])  # [src, dst]
    assert int(to_np(ranks[0][0].status)[0]) == 0
    pitch = row_pitch(H, k)
    # rows: rank s's block for d, into d's receive buffer in source order
    for dd, (epd, *_) in enumerate(ranks):
        off = 0
        for s, (eps, *_) in enumerate(ranks):
            c = int(counts[s, dd])
            b0 = int(counts[s, :dd].sum())
            epd.recv[off * pitch:(off + c) * pitch].copy_(eps.send[b0 * pitch:(b0 + c) * pitch])
            off += c
        epd.compute(off, *_w_of(ranks[dd]))
    # partial rows back to their sources, then the per-token sums
    outs = []
    for s, (eps, *_) in enumerate(ranks):
        off = 0
        for dd, (epd, *_) in enumerate(ranks):
            c = int(counts[s, dd])
            src0 = int(counts[:s, dd].sum())
            eps.ret[off:off + c].copy_(epd.part[src0:src0 + c])
            off += c
        outs.append(to_np(eps.finish(Ts[s])))
    for r in range(W):
        if Ts[r] == 0:
            assert outs[r].shape == (0, H)
            continue
        want, _, _ = moe.expert_mlp(xs[r], inds[r], scores[r].astype(np.float64), g, u, d)
        assert_close(outs[r], want, what=f"a2a EP rank {r}/{W} ({engine})")
    return counts


def _w_of(rank_entry):
    return rank_entry[1], rank_entry[2], rank_entry[3]


@pytest.mark.parametrize("W,engine", [(1, "tc"), (2, "tc"), (3, "mma"), (4, "tc"), (8, "mma"), (8, "tc")])
def test_a2a_expert_parallel_matches_oracle(dev, W, engine):
    Ts = [37 + 11 * r for r in range(W)]
    counts = _run(dev, W, Ts, E=16, H=512, I=256, k=4, engine=engine, seed=W)
    # a token reaches a rank at most once: rows sent <= tokens x min(W, k)
    for r in range(W):
        assert counts[r].sum() <= Ts[r] * min(W, 4)


def test_a2a_rank_without_work_and_empty_rank(dev):
    """One rank's experts get no token, another rank routes no token at all."""
    _run(dev, 4, [40, 0, 25, 33], E=16, H=512, I=256, k=4, engine="tc", seed=5, skip_rank=2)


def test_a2a_deepseek_hidden_size(dev):
    """H 7168 (DeepSeek-V3), I 2048 at a reduced expert count, 2 ranks, sigmoid-style uneven routing."""
    _run(dev, 2, [24, 20], E=8, H=7168, I=2048, k=4, engine="tc", seed=9)
