"""The expert-parallel MoE block over real NCCL collectives, and over the
library's own NVLink peer-memory exchange, one process per GPU (needs at
least two visible GPUs; skipped otherwise).  Each rank checks its tokens'
MoE output against the oracle, eagerly and again from a CUDA graph that
holds the whole block (route, dispatch, plan, experts, partials, combine)
replayed on new inputs, twice (the peer exchange's flags carry the exchange
number across replays)."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path, kind="nccl"):
    from datetime import timedelta

    import torch.distributed as dist

    from b200flash.distributed_experts import ExpertShard
    from b200flash.ep import EPExchange, ExpertParallelMoE, PeerExchange, local_expert_slice
    from helpers import RTOL, ATOL, to_dev, u32_to_dev
    from oracle import affine, moe
    from oracle.fp import round_to

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=120), device_id=dev)
    msg = "ok"
    try:
        T, H, I, k, E = 16, 512, 256, 8, 32
        rng = np.random.default_rng(0)

        def experts(N, K):
            q = affine.quantize(round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16"), 64, 4)
            return q, (u32_to_dev(q[0], dev), to_dev(q[1], "bf16", dev), to_dev(q[2], "bf16", dev))

        (g, gd), (u, ud), (d, dd) = experts(I, H), experts(I, H), experts(H, I)
        wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
        xs = [[round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16") for _ in range(world)]
              for _ in range(3)]
        shard = ExpertShard(rank=rank, world_size=world, total_experts=E)
        ex = PeerExchange() if kind == "p2p" else EPExchange()
        m = ExpertParallelMoE(shard, T, H, I, k, dev, exchange=ex, engine="tc")
        loc = [tuple(local_expert_slice(t, shard) for t in w) for w in (gd, ud, dd)]
        wr_d = to_dev(wr, "bf16", dev)

        def block():
            m.route(wr_d)
            return m.forward(*loc)

        errors = []

        def check(x, tag):
            # records instead of raising, so every rank takes the same collective steps
            oi, osc = moe.route(x, wr.T, k)
            want, _, _ = moe.expert_mlp(x, oi, osc, g, u, d)
            if m.p2p:  # W rows per token, weighted by the ownership mask
                got = (m.out.float().view(T, world, H) * m.mask[:, :, None]).sum(1).cpu().numpy()
                if int(m.p2p_status.item()):
                    errors.append(f"{tag}: peer exchange status {int(m.p2p_status.item())}")
            else:
                got = m.out.float().cpu().numpy()
            bad = np.abs(got - want) > ATOL + RTOL * np.abs(want)
            if bad.any():
                errors.append(f"{tag}: {int(bad.sum())} outside tolerance")
            if int(m.plan_status.item()):
                errors.append(f"{tag}: plan status {int(m.plan_status.item())}")

        m.x.copy_(to_dev(xs[0][rank], "bf16", dev))
        block()
        torch.cuda.synchronize()
        check(xs[0][rank], "eager")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            block()
        for it in (1, 2):
            m.x.copy_(to_dev(xs[it][rank], "bf16", dev))
            graph.replay()
            torch.cuda.synchronize()
            check(xs[it][rank], f"graph replay {it}")
        del graph
        if errors:
            msg = f"rank {rank}: " + "; ".join(errors)
    except Exception as e:  # reported through the file; every rank still leaves the group
        msg = f"rank {rank}: {type(e).__name__}: {e}"
    finally:
        dist.barrier()
        dist.destroy_process_group()
    with open(out_path, "w") as f:
        f.write(msg)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("kind", ["nccl", "p2p"])
def test_ep_block_over_nccl(tmp_path, kind):
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    outs = [str(tmp_path / f"rank{r}.txt") for r in range(world)]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, outs[r], kind)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert [p.exitcode for p in procs] == [0] * world
    for o in outs:
        assert open(o).read() == "ok", open(o).read()
