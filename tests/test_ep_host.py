"""Host side of the expert-parallel MoE on CPU: the routing-segment layout,
the two collectives over a 2-rank gloo group, and the exactness of the
dispatch/combine decomposition (sum over ranks of owner-masked partials
equals the single-process MoE), with the oracle standing in for the expert
kernels on each rank."""

import socket

import numpy as np
import pytest
import torch

from b200flash.distributed_experts import ExpertShard, balanced_placement
from b200flash.ep import RoutingSegment


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("E,W", [(128, 1), (128, 2), (128, 4), (128, 8), (60, 7), (5, 8)])
def test_balanced_placement(E, W):
    """Expert placement over the ExpertShard blocks: a permutation of the
    experts whose blocks keep the ExpertShard sizes (the last rank takes the
    remainder), each rank's expected load within the largest single load of
    the mean, and a load spread no wider than the id blocks' under Zipf
    popularity; one rank (or fewer experts than ranks) keeps the identity."""
    rng = np.random.default_rng(E + W)
    zipf = np.arange(1, E + 1, dtype=np.float64) ** -1.1
    loads = zipf[rng.permutation(E)]  # popularity shuffled over the ids, as the decoder's router bias
    order = balanced_placement(loads, W)
    assert sorted(order) == list(range(E))
    if W == 1 or E < W:
        assert order == list(range(E))
        return
    blocks = [ExpertShard(rank=r, world_size=W, total_experts=E).owned_experts for r in range(W)]
    per_rank = np.array([sum(loads[order[s]] for s in b) for b in blocks])
    assert per_rank.max() - per_rank.mean() <= loads.max() + 1e-12
    ids = np.array([sum(loads[s] for s in b) for b in blocks])
    assert per_rank.max() - per_rank.min() <= ids.max() - ids.min()


def test_routing_segment_layout():
    seg = RoutingSegment(T=64, H=2048, k=8)
    assert seg.row_bytes == 4096
    assert seg.inds_off == 64 * 4096
    assert seg.scores_off == seg.inds_off + 64 * 8 * 4
    assert seg.seg_bytes % seg.row_bytes == 0 and seg.seg_bytes >= seg.scores_off + 64 * 8 * 4
    assert seg.seg_rows == 65
    buf = torch.zeros(3 * seg.seg_bytes, dtype=torch.uint8)
    for r in range(3):
        x, inds, sc = seg.views(buf, r)
        x.fill_(r + 1)
        inds.fill_(10 + r)
        sc.fill_(0.5 * r)
    rows = buf.view(torch.bfloat16).view(3 * seg.seg_rows, 2048)
    for r in range(3):
        x, inds, sc = seg.views(buf, r)
        assert torch.equal(rows[r * seg.seg_rows: r * seg.seg_rows + 64], x)
        assert int(inds[5, 3]) == 10 + r and float(sc[63, 7]) == 0.5 * r
    with pytest.raises(ValueError):
        RoutingSegment(T=4, H=100, k=2)


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist

    from b200flash.ep import EPExchange
    from oracle import affine, moe
    from oracle.fp import round_to

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        ex = EPExchange()
        T, H, I, k, E = 5, 128, 64, 3, 7
        rng = np.random.default_rng(0)

        def experts(N, K):
            return affine.quantize(round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16"), 64, 4)

        g, u, d = experts(I, H), experts(I, H), experts(H, I)
        wr = round_to(rng.normal(0, 0.05, (H, E)).astype(np.float32), "bf16")
        xs = [round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16") for _ in range(world)]
        seg = RoutingSegment(T, H, k)
        send = torch.zeros(seg.seg_bytes, dtype=torch.uint8)
        x, inds, scores = seg.views(send)
        x.copy_(torch.from_numpy(xs[rank]).to(torch.bfloat16))
        oi, osc = moe.route(xs[rank], wr, k)
        inds.copy_(torch.from_numpy(oi))
        scores.copy_(torch.from_numpy(osc.astype(np.float32)))
        recv = torch.empty(world * seg.seg_bytes, dtype=torch.uint8)
        ex.all_gather(recv, send)
        shard = ExpertShard(rank=rank, world_size=world, total_experts=E)
        part = torch.zeros(world * T, H, dtype=torch.float32)
        for r in range(world):
            xr, ir, sr = seg.views(recv, r)
            xr = xr.float().numpy()
            ir = ir.numpy()
            sr = sr.numpy().astype(np.float64)
            _, _, yk = moe.expert_mlp(xr, ir, sr, g, u, d)
            mask = np.vectorize(shard.is_local)(ir)
            part[r * T:(r + 1) * T] = torch.from_numpy((yk * (sr * mask)[..., None]).sum(1))
        out = torch.empty(T, H, dtype=torch.float32)
        ex.reduce_scatter(out, part)
        want, _, _ = moe.expert_mlp(xs[rank], oi, osc, g, u, d)
        err = float(np.abs(out.numpy() - want).max())
        owners = sorted(set(shard.owner_of(int(e)) for e in oi.reshape(-1)))
        with open(out_path, "w") as f:
            f.write(f"{err} {len(owners)}\n")
    finally:
        dist.destroy_process_group()


def test_ep_decomposition_over_gloo(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    outs = [str(tmp_path / f"rank{r}.txt") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, outs[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0] * world
    for o in outs:
        err, n_owners = open(o).read().split()
        assert float(err) < 1e-5, err
        assert int(n_owners) >= 1


def _pack_np(inds, W, E):
    """NumPy statement of b2f_ep_a2a_dispatch's send order: per destination
    d (ascending) the tokens (ascending) with an expert on d."""
    per = E // W
    T = inds.shape[0]
    owner = np.minimum(inds // per, W - 1)
    pos = -np.ones((T, W), np.int64)
    n = 0
    counts = []
    for d in range(W):
        c = 0
        for t in range(T):
            if (owner[t] == d).any():
                pos[t, d] = n
                n += 1
                c += 1
        counts.append(c)
    return pos, counts


def _a2a_rank_main(rank, world, port, out_path):
    import torch.distributed as dist

    from b200flash.ep import EPExchange
    from oracle import affine, moe
    from oracle.fp import round_to

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")
    try:
        ex = EPExchange()
        H, I, k, E = 128, 64, 3, 6
        Ts = [7, 4]
        rng = np.random.default_rng(0)

        def experts(N, K):
            return affine.quantize(round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16"), 64, 4)

        g, u, d = experts(I, H), experts(I, H), experts(H, I)
        xs = [round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16") for T in Ts]
        inds = [np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int64) for T in Ts]
        scs = [rng.uniform(0.1, 1, (T, k)) for T in Ts]
        T = Ts[rank]
        pos, sc = _pack_np(inds[rank], world, E)
        shard = ExpertShard(rank=rank, world_size=world, total_experts=E)
        per = E // world
        # send rows: [x | local ids | scores] as float64 columns
        send = np.zeros((sum(sc), H + 2 * k))
        for t in range(T):
            for dd in range(world):
                if pos[t, dd] >= 0:
                    own = np.minimum(inds[rank][t] // per, world - 1) == dd
                    send[pos[t, dd], :H] = xs[rank][t]
                    send[pos[t, dd], H:H + k] = np.where(own, inds[rank][t] - dd * per, -1)
                    send[pos[t, dd], H + k:] = np.where(own, scs[rank][t], 0)
        rc_t = torch.zeros(world, dtype=torch.int64)
        ex.all_to_all(rc_t, torch.tensor(sc, dtype=torch.int64))
        rc = rc_t.tolist()
        recv = torch.empty(sum(rc), H + 2 * k, dtype=torch.float64)
        ex.all_to_all(recv, torch.from_numpy(send), rc, sc)
        recv = recv.numpy()
        # local experts on the received rows: per row the weighted sum of its local experts
        lo = shard.owned_experts[0]
        loc = (g[0][lo:lo + len(shard.owned_experts)], g[1][lo:], g[2][lo:])
        part = np.zeros((recv.shape[0], H))
        for r in range(recv.shape[0]):
            ids = recv[r, H:H + k].astype(np.int64)
            for j in range(k):
                if ids[j] >= 0:
                    e = lo + ids[j]
                    _, _, yk = moe.expert_mlp(recv[r:r + 1, :H], np.array([[e]]), np.ones((1, 1)), g, u, d)
                    part[r] += recv[r, H + k + j] * yk[0, 0]
        del loc
        ret = torch.empty(sum(sc), H, dtype=torch.float64)
        ex.all_to_all(ret, torch.from_numpy(part), sc, rc)
        ret = ret.numpy()
        out = np.zeros((T, H))
        for t in range(T):
            for dd in range(world):
                if pos[t, dd] >= 0:
                    out[t] += ret[pos[t, dd]]
        want, _, _ = moe.expert_mlp(xs[rank], inds[rank], scs[rank], g, u, d)
        with open(out_path, "w") as f:
            f.write(f"{float(np.abs(out - want).max())} {sum(sc)} {sum(rc)}\n")
    finally:
        dist.destroy_process_group()


def test_a2a_protocol_over_gloo(tmp_path):
    """Counts-then-rows all-to-all, reverse return and per-token sums over a
    2-rank gloo group, with the oracle standing in for the expert kernels."""
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    outs = [str(tmp_path / f"a2a{r}.txt") for r in range(world)]
    procs = [ctx.Process(target=_a2a_rank_main, args=(r, world, port, outs[r])) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0] * world
    for o in outs:
        err, sent, got = open(o).read().split()
        assert float(err) < 1e-9, err
        assert int(sent) > 0
