"""Expert-parallel routed MoE over NCCL (one process per GPU).

Replaces the reference's distributed-expert plan
(``mlx_flash_compress/distributed_experts.py:36-150``: contiguous expert
blocks per rank, ``owner_of``) and the expert-streaming tiers
(``expert_streaming.py``) for the case where every expert is resident in some
GPU's HBM.  Ownership follows ``ExpertShard`` exactly.

Per MoE block, on every rank (T tokens each, attention and router run on the
rank's own tokens):

1. the rank's *routing segment* -- its normalised hidden rows, top-k expert
   ids and scores, laid out back to back in one byte buffer -- is gathered
   onto every rank (``all_gather_into_tensor``: one NCCL call);
2. ``b2f_ep_plan`` sorts the ``W*T*k`` gathered assignments by local expert
   (experts of other ranks skipped) and records each assignment's x row in
   the gathered buffer;
3. the grouped expert kernels run on the local expert shard: the rows are
   copied from the gathered segments into expert-sorted order
   (``b2f_moe_gather_rows``) for the tcgen05 GEMM, or read in place through
   the x-row index by the register GEMV;
4. ``b2f_ep_combine_partial`` forms every gathered token's score-weighted sum
   over its local experts;
5. ``reduce_scatter_tensor`` (sum) returns to each rank the sum over ranks of
   its own tokens' partials -- the complete MoE output.

All buffers are allocated once, so the block (collectives included) can be
captured in a CUDA graph.  No TMA multicast is used anywhere on this path.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _capi
from ._capi import call, ptr, require_cuda, stream_of
from .distributed_experts import ExpertShard


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


class RoutingSegment:
    """Byte layout of one rank's routing segment (T tokens, hidden H, top-k).

    ``[0, T*2H)``: bf16 x rows (row pitch ``2H`` bytes); ``inds_off``: int32
    ``[T, k]`` expert ids; ``scores_off``: float32 ``[T, k]``.  The segment is
    padded to a whole number of x rows so gathered segments stay one bf16
    matrix of ``W * seg_rows`` rows.
    """

    def __init__(self, T: int, H: int, k: int):
        if H % 8:
            raise ValueError("hidden size must be a multiple of 8")
        self.T, self.H, self.k = T, H, k
        self.row_bytes = 2 * H
        self.inds_off = T * self.row_bytes
        self.scores_off = self.inds_off + 4 * T * k
        self.seg_bytes = _align(self.scores_off + 4 * T * k, self.row_bytes)
        self.seg_rows = self.seg_bytes // self.row_bytes

    def views(self, buf: torch.Tensor, r: int = 0):
        """(x bf16 [T,H], inds int32 [T,k], scores f32 [T,k]) views of segment r of ``buf``."""
        base = r * self.seg_bytes
        T, H, k = self.T, self.H, self.k
        x = buf[base: base + T * self.row_bytes].view(torch.bfloat16).view(T, H)
        inds = buf[base + self.inds_off: base + self.inds_off + 4 * T * k].view(torch.int32).view(T, k)
        scores = buf[base + self.scores_off: base + self.scores_off + 4 * T * k].view(torch.float32).view(T, k)
        return x, inds, scores


class EPExchange:
    """The two collectives of the expert-parallel MoE over a process group.

    NCCL groups use ``all_gather_into_tensor`` / ``reduce_scatter_tensor``
    directly.  Gloo has no reduce-scatter, so on a CPU group the combine is an
    ``all_reduce`` followed by taking this rank's slice (same result).
    """

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.backend = dist.get_backend(group)

    def all_gather(self, recv: torch.Tensor, send: torch.Tensor):
        dist.all_gather_into_tensor(recv, send, group=self.group)

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None):
        """``all_to_all_single`` over the group's first dimension (splits in rows)."""
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor):
        if self.backend == "nccl":
            dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=self.group)
        else:
            tmp = inp.clone()
            dist.all_reduce(tmp, op=dist.ReduceOp.SUM, group=self.group)
            out.copy_(tmp.view(self.world, *out.shape)[self.rank])


class PeerExchange:
    """The two exchanges of the expert-parallel MoE done by this library's
    kernels over NVLink peer memory (``b2f_ep_p2p_*``) instead of NCCL
    collectives: every rank holds one shared region (routing segments of all
    ranks, the combine rows of its own tokens, the exchange flags), mapped
    into every other rank's process by CUDA IPC.  The process group only
    carries the one-time exchange of the IPC handles; no NCCL call runs in a
    decode step.  One process per GPU on one node, peer access between every
    pair of GPUs (NVSwitch)."""

    kind = "p2p"

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def map_region(self, nbytes: int, device):
        """A zeroed region of ``nbytes`` on this rank, mapped on every rank.
        Returns (own region, int64 device table of the W regions' addresses in
        this process, a handle that unmaps the peers' regions when released).

        Each peer region is opened by ``b2f_ipc_import`` with THIS rank's
        device current, so the mapping belongs to the device whose kernels
        store into it (with peer access enabled); a mapping opened under the
        owner's device index would leave this device without peer access."""
        device = torch.device(device)
        for r in range(torch.cuda.device_count()):
            if r != device.index and not torch.cuda.can_device_access_peer(device, r):
                raise RuntimeError(f"peer exchange: GPU {device.index} cannot access GPU {r}")
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)
        lib = _capi.lib()
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        _capi.check(lib.b2f_ipc_export(ptr(buf), handle, ctypes.addressof(off)), "b2f_ipc_export")
        shared = [None] * self.world
        dist.all_gather_object(shared, (handle.raw, off.value), group=self.group)
        addrs, mapped = [], _PeerMappings()
        with torch.cuda.device(device):
            for r, (h, o) in enumerate(shared):
                if r == self.rank:
                    addrs.append(buf.data_ptr())
                    continue
                base = ctypes.c_void_p(0)
                _capi.check(lib.b2f_ipc_import(ctypes.create_string_buffer(h, 64), ctypes.addressof(base)),
                            "b2f_ipc_import")
                mapped.bases.append(base.value)
                addrs.append(base.value + o)
        peers = torch.tensor(addrs, dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        # every region is zeroed and mapped before any rank's first exchange
        dist.barrier(group=self.group)
        return buf, peers, mapped


class _PeerMappings:
    """Peer regions opened by b2f_ipc_import; unmapped when released."""

    def __init__(self):
        self.bases = []

    def __del__(self):
        try:
            lib = _capi.lib()
            for b in self.bases:
                lib.b2f_ipc_close(ctypes.c_void_p(b))
        except Exception:
            pass
        self.bases = []


class LocalPeerGroup:
    """W ranks' shared regions on ONE device (the single-GPU emulation the
    tests use): ``exchange(r)`` is rank r's view.  Each rank's kernels store
    into the other emulated ranks' regions exactly as into a peer GPU's;
    the caller runs the phases so that every wait finds its flags raised
    (all dispatches before any dispatch wait, all combines before any
    combine wait)."""

    def __init__(self, W: int, device):
        self.W = W
        self.device = torch.device(device)
        self.bufs = None
        self.peers = None

    def exchange(self, rank: int):
        grp = self

        class _Ex:
            kind = "p2p"
            world = grp.W

            def __init__(self):
                self.rank = rank

            def map_region(self, nbytes, device):
                if grp.bufs is None:
                    grp.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=grp.device) for _ in range(grp.W)]
                    grp.peers = torch.tensor([b.data_ptr() for b in grp.bufs], dtype=torch.int64, device=grp.device)
                return grp.bufs[rank], grp.peers, grp.bufs

        return _Ex()


class ExpertParallelMoE:
    """Buffers and launches of the expert-parallel MoE block for one rank.

    ``shard``: this rank's ``ExpertShard``.  ``T``: tokens per rank per call
    (fixed; the buffers are sized for it).  The caller writes the normalised
    hidden state into ``self.x`` (a view into the send segment), calls
    :meth:`route`, then :meth:`forward` with the layer's local expert weights
    ``(wq, scales, biases)`` stacked over the ``len(shard.owned_experts)``
    local experts; the result lands in ``self.out`` (bf16 ``[T, H]``).
    """

    def __init__(self, shard: ExpertShard, T: int, hidden: int, inter: int, top_k: int, device,
                 bits: int = 4, group_size: int = 64, exchange: EPExchange = None, engine: str = "auto",
                 tile: int = None):
        self.shard = shard
        self.W = shard.world_size
        self.rank = shard.rank
        owned = shard.owned_experts
        if not owned or owned != list(range(owned[0], owned[0] + len(owned))):
            raise ValueError("expert parallelism needs a non-empty contiguous expert block per rank")
        self.e_begin, self.e_count, self.e_total = owned[0], len(owned), shard.total_experts
        self.T, self.H, self.I, self.k = T, hidden, inter, top_k
        self.bits, self.gs = bits, group_size
        self.dev = dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("ExpertParallelMoE runs on CUDA devices only")
        if exchange is not None and exchange.world != self.W:
            raise ValueError("exchange world size differs from the shard's")
        self.exchange = exchange
        self.seg = seg = RoutingSegment(T, hidden, top_k)
        self.p2p = getattr(exchange, "kind", None) == "p2p"
        if self.p2p:
            so, co = ctypes.c_int64(0), ctypes.c_int64(0)
            nbytes = int(_capi.lib().b2f_ep_p2p_region_bytes(self.W, T, hidden, seg.seg_bytes,
                                                              ctypes.addressof(so), ctypes.addressof(co)))
            if nbytes <= 0:
                raise ValueError("peer exchange: unsupported sizes")
            self.region, self.peers, self._mapped = exchange.map_region(nbytes, dev)
            self.seg_off, self.comb_off, self.flags_off = so.value, co.value, 0
            self.recv = self.region[so.value: so.value + self.W * seg.seg_bytes]
            self.send = self.recv[self.rank * seg.seg_bytes: (self.rank + 1) * seg.seg_bytes]
            # combine rows [T][W][H] and their weights (1 where rank d owns one
            # of token m's experts): b2f_combine_rmsnorm with k = W sums them
            self.comb = self.region[co.value: co.value + T * self.W * hidden * 2].view(torch.bfloat16).view(
                T * self.W, hidden)
            self.mask = torch.zeros(T, self.W, dtype=torch.float32, device=dev)
            self.ctl = torch.zeros(4, dtype=torch.int32, device=dev)
            self.p2p_status = torch.zeros(1, dtype=torch.int32, device=dev)
        else:
            self.send = torch.zeros(seg.seg_bytes, dtype=torch.uint8, device=dev)
            self.recv = self.send if self.W == 1 else torch.zeros(self.W * seg.seg_bytes, dtype=torch.uint8,
                                                                  device=dev)
        self.x, self.inds, self.scores = seg.views(self.send)
        self.G = self.W * T
        self.A = self.G * top_k
        A = self.A
        self.x_row = torch.zeros(A, dtype=torch.int32, device=dev)
        self.wts = torch.zeros(A, dtype=torch.float32, device=dev)
        self.local = torch.full((A,), -1, dtype=torch.int32, device=dev)
        if engine == "auto":
            if bits == 4 and group_size == 64 and hidden % 128 == 0 and inter % 128 == 0:
                engine = "mma"
            else:
                engine = "tc_gather" if T * top_k >= self.e_count and group_size == 64 else "gemv"
        if engine not in ("tc", "tc_gather", "gemv", "mma"):
            raise ValueError(f"unknown expert engine {engine!r}")
        if engine == "tc" and ((hidden // 64) % 2 or (inter // 64) % 2):
            engine = "tc_gather"  # the sorted-row kernel copies scales two groups at a time
        if engine == "mma" and (bits != 4 or group_size != 64 or hidden % 128 or inter % 128):
            engine = "tc_gather"  # register-dequant MMA: 4-bit, group 64, 128-wide K chunks
        self.engine = engine
        if tile is None:
            if engine == "tc_gather":
                tile = 32
            elif engine == "mma":
                tile = 16
            else:
                tile = min(256, max(16, (T + 15) // 16 * 16)) if engine != "gemv" else 16
        self.tile = tile
        self.plan_bytes = int(_capi.lib().b2f_moe_plan_workspace_bytes(A, self.e_count, tile))
        self.plan_ws = torch.empty(max(self.plan_bytes, 16), dtype=torch.uint8, device=dev)
        self.plan_status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.gates = torch.empty(T, self.e_total, dtype=torch.float32, device=dev)
        self.hh = torch.empty(A, inter, dtype=torch.bfloat16, device=dev)
        self.xs = torch.empty(A, hidden, dtype=torch.bfloat16, device=dev) if engine == "tc" else None
        self.y = torch.empty(A, hidden, dtype=torch.bfloat16, device=dev)
        self.part = torch.empty(self.G, hidden, dtype=torch.bfloat16, device=dev)
        # stream-K workspace of the packed expert GEMM (zeroed once; left zeroed)
        self.sk_bytes = int(_capi.lib().b2f_mma_streamk_workspace_bytes()) if engine == "mma" else 0
        self.sk_ws = torch.zeros(max(self.sk_bytes, 256), dtype=torch.uint8, device=dev)
        if self.p2p:
            self.out = self.comb
        else:
            self.out = self.part if self.W == 1 else torch.empty(T, hidden, dtype=torch.bfloat16, device=dev)

    # -- phases (the single-GPU multi-rank emulation in the tests drives them one by one)
    def route(self, wr: torch.Tensor, bias: torch.Tensor = None, renorm: bool = True):
        """Softmax top-k routing of ``self.x`` into the send segment."""
        call("b2f_moe_route_topk", ptr(self.x), self.T, self.H, ptr(wr), ptr(bias), self.e_total, self.k,
             int(renorm), ptr(self.gates), ptr(self.inds), ptr(self.scores), stream_of(self.dev))

    def dispatch(self):
        if self.p2p:
            self.dispatch_send()  # the plan in compute() waits for every rank's dispatch
        elif self.W > 1:
            self.exchange.all_gather(self.recv, self.send)

    # peer exchange phases (forward() runs them in order; the one-GPU
    # emulation runs every rank's send before any rank's wait)
    def dispatch_send(self):
        st = stream_of(self.dev)
        call("b2f_ep_p2p_dispatch", ptr(self.send), self.seg.seg_bytes, ptr(self.peers), self.seg_off,
             self.flags_off, self.rank, self.W, ptr(self.inds), self.T, self.k, self.e_total, ptr(self.mask),
             ptr(self.ctl), ptr(self.p2p_status), st)

    def dispatch_wait(self):
        call("b2f_ep_p2p_wait", ptr(self.region), self.flags_off, 0, self.W, ptr(self.ctl), ptr(self.p2p_status),
             stream_of(self.dev))

    def combine_wait(self):
        call("b2f_ep_p2p_wait", ptr(self.region), self.flags_off, 1, self.W, ptr(self.ctl), ptr(self.p2p_status),
             stream_of(self.dev))

    @property
    def combine_k(self) -> int:
        """Rows per token of ``out`` (W with the peer exchange: sum them
        weighted by ``mask``; else 1, already summed)."""
        return self.W if self.p2p else 1

    def compute(self, gate, up, down, packed=None):
        """Plan over the gathered assignments, local experts, weighted partial
        sums.  ``packed``: (gate/up tiles of mat 2 each, down tiles of mat 1)
        from b2f_mma_repack of the local experts, for the warp-MMA engine with
        16-token tiles: one bulk copy per staged tile, stream-K ranges."""
        seg, st = self.seg, stream_of(self.dev)
        if self.p2p:
            # the plan first waits for the W dispatch flags of this exchange
            call("b2f_ep_p2p_plan", ptr(self.region), self.seg_off, self.flags_off, seg.seg_bytes, seg.row_bytes,
                 seg.inds_off, seg.scores_off, self.W, self.T, self.k, self.e_begin, self.e_count, self.e_total,
                 self.tile, ptr(self.x_row), ptr(self.wts), ptr(self.local), ptr(self.plan_ws), self.plan_bytes,
                 ptr(self.plan_status), ptr(self.ctl), ptr(self.p2p_status), st)
        else:
            call("b2f_ep_plan", ptr(self.recv), seg.seg_bytes, seg.row_bytes, seg.inds_off, seg.scores_off, self.W,
                 self.T, self.k, self.e_begin, self.e_count, self.e_total, self.tile, ptr(self.x_row),
                 ptr(self.wts), ptr(self.local), ptr(self.plan_ws), self.plan_bytes, ptr(self.plan_status), st)
        gw, gs_, gb = gate
        uw, us, ub = up
        dw, ds, db = down
        if packed is not None:
            if self.engine != "mma" or self.tile != 16:
                raise ValueError("packed expert tiles run on the warp-MMA engine with 16-token tiles")
            pg, pu, pd = packed
            sk = ptr(self.sk_ws) if self.sk_bytes else 0
            call("b2f_gather_qgemm_affine_mma_packed", ptr(self.recv), self.H, ptr(self.x_row), 1, 0, self.A,
                 self.e_count, ptr(pg), ptr(pu), self.I, self.H, self.bits, self.gs, self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.hh), self.I, 1, sk, self.sk_bytes, 0, st)
            call("b2f_gather_qgemm_affine_mma_packed", ptr(self.hh), self.I, 0, 1, 1, self.A, self.e_count,
                 ptr(pd), 0, self.H, self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws), self.plan_bytes,
                 ptr(self.y), self.H, 0, sk, self.sk_bytes, 0, st)
        elif self.engine == "mma":
            call("b2f_gather_qgemm_affine_mma", ptr(self.recv), self.H, ptr(self.x_row), 1, 0, self.A, self.e_count,
                 ptr(gw), ptr(gs_), ptr(gb), ptr(uw), ptr(us), ptr(ub), self.I, self.H, self.bits, self.gs, self.tile,
                 ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), self.I, 1, st)
            call("b2f_gather_qgemm_affine_mma", ptr(self.hh), self.I, 0, 1, 1, self.A, self.e_count, ptr(dw),
                 ptr(ds), ptr(db), 0, 0, 0, self.H, self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.y), self.H, 0, st)
        elif self.engine == "tc":
            call("b2f_moe_gather_rows", ptr(self.recv), self.H, ptr(self.x_row), 1, self.A, self.e_count, self.tile,
                 ptr(self.plan_ws), self.plan_bytes, self.H, ptr(self.xs), self.H, st)
            call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.xs), self.H, self.A, self.e_count, ptr(gw), ptr(gs_),
                 ptr(gb), ptr(uw), ptr(us), ptr(ub), self.I, self.H, self.bits, self.gs, self.tile,
                 ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), self.I, 1, st)
            call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.hh), self.I, self.A, self.e_count, ptr(dw), ptr(ds),
                 ptr(db), 0, 0, 0, self.H, self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.y), self.H, 0, st)
        else:
            fn = "b2f_gather_qgemm_affine_tcgen05" if self.engine == "tc_gather" else "b2f_gather_qgemv_affine"
            call(fn, ptr(self.recv), self.H, ptr(self.x_row), 1, self.A, self.e_count, ptr(gw), ptr(gs_), ptr(gb),
                 ptr(uw), ptr(us), ptr(ub), self.I, self.H, self.bits, self.gs, self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.hh), self.I, st)
            call(fn, ptr(self.hh), self.I, 0, 1, self.A, self.e_count, ptr(dw), ptr(ds), ptr(db), 0, 0, 0, self.H,
                 self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws), self.plan_bytes, ptr(self.y), self.H, st)
        if self.p2p:
            call("b2f_ep_p2p_combine", ptr(self.y), self.H, ptr(self.wts), ptr(self.local), self.T, self.k, self.H,
                 ptr(self.peers), self.comb_off, self.flags_off, self.rank, self.W, ptr(self.ctl), st)
            return
        call("b2f_ep_combine_partial", ptr(self.y), self.H, ptr(self.wts), ptr(self.local), self.G, self.k,
             self.H, ptr(self.part), self.H, st)

    def combine(self):
        if self.p2p:
            self.combine_wait()
        elif self.W > 1:
            self.exchange.reduce_scatter(self.out, self.part)

    def forward(self, gate, up, down, packed=None, wait_combine: bool = True) -> torch.Tensor:
        """``wait_combine=False`` (peer exchange): the caller completes the
        combine with :meth:`combine_rmsnorm`, which waits for the rows itself."""
        self.dispatch()
        self.compute(gate, up, down, packed)
        if wait_combine or not self.p2p:
            self.combine()
        return self.out

    def combine_rmsnorm(self, resid, weight, eps, resid_out, norm_out):
        """Peer exchange: once every rank's combine rows have arrived,
        ``resid_out = resid + sum_d mask * rows`` and ``norm_out = RMSNorm`` (one
        launch); the NCCL form: b2f_combine_rmsnorm over the summed output."""
        st = stream_of(self.dev)
        if self.p2p:
            call("b2f_ep_p2p_combine_rmsnorm", ptr(resid), ptr(self.region), self.comb_off, self.flags_off,
                 ptr(self.mask), self.T, self.W, ptr(weight), eps, self.H, ptr(resid_out), ptr(norm_out),
                 ptr(self.ctl), ptr(self.p2p_status), st)
        else:
            call("b2f_combine_rmsnorm", ptr(resid), ptr(self.out), 0, self.T, 1, ptr(weight), eps, self.H,
                 ptr(resid_out), ptr(norm_out), st)

    def check(self):
        """Synchronising check that every gathered expert id was in range (and,
        with the peer exchange, that no wait ran out)."""
        if int(self.plan_status.item()):
            raise IndexError("expert index out of range in the gathered routing")
        if self.p2p:
            st = int(self.p2p_status.item())
            if st == _capi.B2F_ERR_TIMEOUT:
                raise TimeoutError("peer exchange: a rank's flags did not arrive within the wait limit")
            if st:
                raise IndexError("expert index out of range in this rank's routing")

    @property
    def launches_per_block(self) -> int:
        """route, plan, (row gather), gate/up, down, partial; the collectives
        are NCCL's, or with the peer exchange the dispatch (the plan and the
        owner's combine + RMSNorm wait for the flags themselves)."""
        return (6 if self.engine == "tc" else 5) + (1 if self.p2p else 0)


def local_expert_slice(w: torch.Tensor, shard: ExpertShard) -> torch.Tensor:
    """Rows of a stacked ``[E, ...]`` expert tensor that ``shard`` owns."""
    owned = shard.owned_experts
    return w[owned[0]: owned[-1] + 1]


def ep_moe_block(x: torch.Tensor, wr: torch.Tensor, gate, up, down, top_k: int, shard: ExpertShard,
                 exchange: EPExchange = None, bias=None, renorm=True, group_size: int = 64, bits: int = 4):
    """One-shot expert-parallel MoE block: ``sum_k score_k * expert_k(x)`` for this rank's tokens.

    ``gate``/``up``/``down``: ``(wq, scales, biases)`` of this rank's local
    experts only.  Builds the buffers on every call; a decode loop keeps one
    :class:`ExpertParallelMoE` instead.
    """
    dev = require_cuda(x, wr)
    T, H = x.shape
    inter = gate[0].shape[1]
    moe = ExpertParallelMoE(shard, T, H, inter, top_k, dev, bits, group_size, exchange)
    moe.x.copy_(x)
    moe.route(wr.contiguous(), None if bias is None else bias.to(torch.float32).contiguous(), renorm)
    out = moe.forward(gate, up, down)
    return out.clone(), moe.inds.clone(), moe.scores.clone()
