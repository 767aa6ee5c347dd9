"""Expert-parallel MoE with a variable-split all-to-all (prefill-sized batches).

The expert-parallel plan of the reference (``mlx_flash_compress/
distributed_experts.py:36-150``: ``ExpertShard`` blocks, ``owner_of``) with
every expert resident on its owner GPU.  Per MoE block, on each rank:

1. ``b2f_ep_a2a_dispatch``: each of the rank's tokens goes once to every rank
   that owns at least one of its k experts, as one row
   ``[bf16 hidden row][int32 local expert ids k][float32 scores k]`` in a send
   buffer grouped by destination rank (``pos[t, d]`` remembers where);
2. counts first: ``all_to_all_single`` of the per-destination row counts, read
   on the host (the split sizes NCCL needs), then the rows themselves in one
   ``all_to_all_single`` with those byte splits;
3. ``b2f_ep_a2a_plan``: counting sort of the received rows' (row, local
   expert) assignments by local expert;
4. the local experts: the received rows gathered into expert order
   (``b2f_moe_gather_rows``), then the tcgen05 grouped GEMMs with the SwiGLU
   fused into gate/up (``b2f_sorted_qgemm_affine_tcgen05``), or warp MMA at
   decode density;
5. ``b2f_ep_combine_partial``: per received row the score-weighted sum of its
   local experts' outputs;
6. ``all_to_all_single`` back with the reverse splits, and
   ``b2f_ep_a2a_combine``: each token's output is the sum of the partial rows
   its owner ranks returned (fixed rank order) plus the residual.

Only rows a rank computed travel back (no dense ``[W*T, H]`` partials), and
a token crosses to a peer once whatever number of its experts the peer owns.
The host reads the counts once per block, so this path is not captured in a
CUDA graph; the decode step's all-gather path (``ep.ExpertParallelMoE``) is.
No TMA multicast is used; NCCL moves the rows.
"""

import torch

from . import _capi
from ._capi import call, ptr, require_cuda, stream_of
from .distributed_experts import ExpertShard


def row_pitch(H: int, k: int) -> int:
    """Bytes per dispatched row: the bf16 hidden row, k int32 ids, k float32 scores, 16-byte aligned."""
    return int(_capi.lib().b2f_ep_a2a_row_pitch(H, k))


class ExpertParallelA2A:
    """Buffers and launches of the all-to-all expert-parallel MoE for one rank.

    ``T_max``: most tokens this rank routes per call; every rank receives at
    most ``W * T_max`` rows.  ``forward(x, inds, scores, gate, up, down)``
    takes the rank's bf16 ``[T, H]`` rows with their global top-k ids and
    scores and this rank's local experts ``(wq, scales, biases)`` stacked over
    ``len(shard.owned_experts)``; it returns bf16 ``[T, H]`` (plus
    ``residual`` when given).
    """

    def __init__(self, shard: ExpertShard, T_max: int, hidden: int, inter: int, top_k: int, device, bits: int = 4,
                 group_size: int = 64, exchange=None, engine: str = "auto", tile: int = None):
        self.shard = shard
        self.W, self.rank = shard.world_size, shard.rank
        owned = shard.owned_experts
        if not owned or owned != list(range(owned[0], owned[0] + len(owned))):
            raise ValueError("expert parallelism needs a non-empty contiguous expert block per rank")
        self.e_begin, self.e_count, self.e_total = owned[0], len(owned), shard.total_experts
        self.T_max, self.H, self.I, self.k = int(T_max), int(hidden), int(inter), int(top_k)
        self.bits, self.gs = bits, group_size
        self.dev = dev = torch.device(device)
        if dev.type != "cuda":
            raise RuntimeError("ExpertParallelA2A runs on CUDA devices only")
        if exchange is not None and exchange.world != self.W:
            raise ValueError("exchange world size differs from the shard's")
        self.exchange = exchange
        self.pitch = row_pitch(hidden, top_k)
        cap_send = self.T_max * min(self.W, top_k)
        self.R_max = self.W * self.T_max
        self.send = torch.empty(cap_send * self.pitch, dtype=torch.uint8, device=dev)
        self.recv = self.send if self.W == 1 else torch.empty(self.R_max * self.pitch, dtype=torch.uint8, device=dev)
        self.pos = torch.empty(self.T_max * self.W, dtype=torch.int32, device=dev)
        self.send_counts = torch.zeros(self.W, dtype=torch.int32, device=dev)
        self.recv_counts = torch.zeros(self.W, dtype=torch.int32, device=dev)
        self.status = torch.zeros(2, dtype=torch.int32, device=dev)
        A = self.R_max * top_k
        self.A_max = A
        self.x_row = torch.empty(A, dtype=torch.int32, device=dev)
        self.wts = torch.empty(A, dtype=torch.float32, device=dev)
        self.local = torch.empty(A, dtype=torch.int32, device=dev)
        dense = A >= 16 * self.e_count
        if engine == "auto":
            engine = "tc" if group_size == 64 and (hidden // 64) % 2 == 0 and (inter // 64) % 2 == 0 and dense \
                else ("mma" if bits == 4 and group_size == 64 and hidden % 128 == 0 and inter % 128 == 0 else "tc")
        if engine not in ("tc", "mma"):
            raise ValueError(f"unknown expert engine {engine!r}")
        self.engine = engine
        if tile is None:
            # tcgen05 at prefill density: each dequantized weight tile serves up
            # to 256 tokens (the dequantizing warps bound this GEMM; measured
            # on the DeepSeek-V3-shaped layer: tiles 64 / 128 / 256 give
            # 185 / 300 / 336 TFLOP/s)
            tile = 16 if engine == "mma" else (256 if A >= 64 * self.e_count else 128)
        self.tile = int(tile)
        self.plan_bytes = int(_capi.lib().b2f_moe_plan_workspace_bytes(A, self.e_count, self.tile))
        self.plan_ws = torch.empty(max(self.plan_bytes, 16), dtype=torch.uint8, device=dev)
        self.xs = torch.empty(A, hidden, dtype=torch.bfloat16, device=dev) if engine == "tc" else None
        self.hh = torch.empty(A, inter, dtype=torch.bfloat16, device=dev)
        self.y = torch.empty(A, hidden, dtype=torch.bfloat16, device=dev)
        self.part = torch.empty(self.R_max, hidden, dtype=torch.bfloat16, device=dev)
        self.ret = self.part if self.W == 1 else torch.empty(cap_send, hidden, dtype=torch.bfloat16, device=dev)
        self.last_counts = None

    # -- phases (the one-GPU multi-rank emulation in the tests drives them one by one)
    def pack(self, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor):
        """Rows for every destination rank into ``send`` (counts in ``send_counts``)."""
        T = x.shape[0]
        if T > self.T_max:
            raise ValueError(f"{T} tokens exceed T_max={self.T_max}")
        call("b2f_ep_a2a_dispatch", ptr(x), x.stride(0), ptr(inds), ptr(scores), T, self.k, self.W, self.e_total,
             self.H, ptr(self.send), self.send.numel(), ptr(self.pos), ptr(self.send_counts), ptr(self.status),
             stream_of(self.dev))

    def exchange_rows(self):
        """Counts first (read on the host: NCCL's split sizes), then the rows.
        Returns (rows sent per rank, rows received per rank) as lists."""
        if self.W > 1:
            self.exchange.all_to_all(self.recv_counts, self.send_counts)
        else:
            self.recv_counts.copy_(self.send_counts)
        counts = torch.stack([self.send_counts, self.recv_counts]).cpu()
        sc, rc = counts[0].tolist(), counts[1].tolist()
        if self.W > 1:
            p = self.pitch
            self.exchange.all_to_all(self.recv[: sum(rc) * p], self.send[: sum(sc) * p], [c * p for c in rc],
                                     [c * p for c in sc])
        self.last_counts = (sc, rc)
        return sc, rc

    def dispatch(self, x: torch.Tensor, inds: torch.Tensor, scores: torch.Tensor):
        self.pack(x, inds, scores)
        return self.exchange_rows()

    def compute(self, R: int, gate, up, down):
        """Plan over the R received rows, local experts, per-row partial sums."""
        st = stream_of(self.dev)
        A = R * self.k
        if A == 0:
            return
        call("b2f_ep_a2a_plan", ptr(self.recv), R, self.H, self.k, self.e_count, self.tile, ptr(self.x_row),
             ptr(self.wts), ptr(self.local), ptr(self.plan_ws), self.plan_bytes, ptr(self.status[1:]), st)
        gw, gs_, gb = gate
        uw, us, ub = up
        dw, ds, db = down
        ldx = self.pitch // 2  # the received rows as a bf16 matrix
        if self.engine == "tc":
            call("b2f_moe_gather_rows", ptr(self.recv), ldx, ptr(self.x_row), 1, A, self.e_count, self.tile,
                 ptr(self.plan_ws), self.plan_bytes, self.H, ptr(self.xs), self.H, st)
            call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.xs), self.H, A, self.e_count, ptr(gw), ptr(gs_), ptr(gb),
                 ptr(uw), ptr(us), ptr(ub), self.I, self.H, self.bits, self.gs, self.tile, ptr(self.plan_ws),
                 self.plan_bytes, ptr(self.hh), self.I, 1, st)
            call("b2f_sorted_qgemm_affine_tcgen05", ptr(self.hh), self.I, A, self.e_count, ptr(dw), ptr(ds), ptr(db),
                 0, 0, 0, self.H, self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws), self.plan_bytes,
                 ptr(self.y), self.H, 0, st)
        else:
            call("b2f_gather_qgemm_affine_mma", ptr(self.recv), ldx, ptr(self.x_row), 1, 0, A, self.e_count, ptr(gw),
                 ptr(gs_), ptr(gb), ptr(uw), ptr(us), ptr(ub), self.I, self.H, self.bits, self.gs, self.tile,
                 ptr(self.plan_ws), self.plan_bytes, ptr(self.hh), self.I, 1, st)
            call("b2f_gather_qgemm_affine_mma", ptr(self.hh), self.I, 0, 1, 1, A, self.e_count, ptr(dw), ptr(ds),
                 ptr(db), 0, 0, 0, self.H, self.I, self.bits, self.gs, self.tile, ptr(self.plan_ws), self.plan_bytes,
                 ptr(self.y), self.H, 0, st)
        call("b2f_ep_combine_partial", ptr(self.y), self.H, ptr(self.wts), ptr(self.local), R, self.k, self.H,
             ptr(self.part), self.H, st)

    def return_rows(self, sc, rc):
        """The partial rows back to their source ranks (reverse splits)."""
        if self.W > 1:
            self.exchange.all_to_all(self.ret[: sum(sc)], self.part[: sum(rc)], sc, rc)

    def finish(self, T: int, residual: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
        """Each token's sum of the partial rows its owner ranks returned (+ residual)."""
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.dev)
        call("b2f_ep_a2a_combine", ptr(self.ret), self.H, ptr(self.pos), T, self.W, self.H,
             ptr(residual) if residual is not None else 0, ptr(out), self.H, stream_of(self.dev))
        return out

    def combine(self, T: int, sc, rc, residual: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
        self.return_rows(sc, rc)
        return self.finish(T, residual, out)

    def forward(self, x, inds, scores, gate, up, down, residual=None, out=None) -> torch.Tensor:
        require_cuda(x, inds, scores)
        sc, rc = self.dispatch(x, inds, scores)
        self.compute(sum(rc), gate, up, down)
        return self.combine(x.shape[0], sc, rc, residual, out)

    def check(self):
        """Synchronising check of the dispatch / plan status words (expert ids in range)."""
        if self.status.any().item():
            raise IndexError("expert index out of range in the routing")
