"""Expert-parallel partition -- drop-in for ``mlx_flash_compress/distributed_experts.py``.

The reference only plans the sharding (``distributed_experts.py:36-150``);
here the same ownership rule drives the NCCL expert-parallel MoE in
``b200flash.ep``.  Ownership: rank ``r`` of ``W`` owns the contiguous block
``[r*floor(E/W), (r+1)*floor(E/W))`` and the last rank also takes the
remainder; ``owner_of(e) = min(e // floor(E/W), W-1)`` (0 when E < W).
``DistributedConfig.from_env`` reads the reference's ``MLX_WORLD_SIZE`` /
``MLX_RANK`` and falls back to torchrun's ``WORLD_SIZE`` / ``RANK``.
"""

import os
from dataclasses import dataclass, field


@dataclass
class ExpertShard:
    """Which experts this rank owns (distributed_experts.py:36-80)."""

    rank: int = 0
    world_size: int = 1
    total_experts: int = 60
    owned_experts: list = field(default_factory=list)

    def __post_init__(self):
        if not self.owned_experts:
            self.owned_experts = self._compute_owned()

    def _block(self) -> int:
        return self.total_experts // self.world_size

    def _compute_owned(self) -> list:
        per = self._block()
        start = self.rank * per
        end = self.total_experts if self.rank == self.world_size - 1 else start + per
        return list(range(start, end))

    def is_local(self, expert_id: int) -> bool:
        return expert_id in set(self.owned_experts)

    def owner_of(self, expert_id: int) -> int:
        per = self._block()
        if per == 0:
            return 0
        return min(expert_id // per, self.world_size - 1)

    def owner_table(self) -> list:
        """``owner_of`` for every expert id (the table the EP dispatch uses)."""
        return [self.owner_of(e) for e in range(self.total_experts)]

    def stats(self) -> dict:
        owned = self.owned_experts
        return {
            "rank": self.rank,
            "world_size": self.world_size,
            "total_experts": self.total_experts,
            "local_experts": len(owned),
            "expert_range": f"{owned[0]}-{owned[-1]}" if owned else "none",
            "memory_fraction": len(owned) / max(self.total_experts, 1),
        }


@dataclass
class DistributedConfig:
    """Distributed settings (distributed_experts.py:83-106); backend here is NCCL."""

    world_size: int = 1
    rank: int = 0
    backend: str = "nccl"
    link_bandwidth_gbps: float = 7200.0  # NVLink 5: 900 GB/s per direction

    @classmethod
    def from_env(cls) -> "DistributedConfig":
        ws = os.environ.get("MLX_WORLD_SIZE", os.environ.get("WORLD_SIZE", "1"))
        rk = os.environ.get("MLX_RANK", os.environ.get("RANK", "0"))
        return cls(world_size=int(ws), rank=int(rk))

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def plan_expert_distribution(num_experts: int, num_layers: int, world_size: int,
                             expert_size_mb: float = 50.0, hidden_dim: int = 4096, top_k: int = 4,
                             link_bandwidth_gbps: float = 7200.0) -> dict:
    """Memory / traffic estimate of a contiguous expert partition (distributed_experts.py:109-150)."""
    per = num_experts // world_size
    rem = num_experts % world_size
    total_gb = num_experts * num_layers * expert_size_mb / 1024
    per_gb = per * num_layers * expert_size_mb / 1024
    non_local = (world_size - 1) / world_size
    comm = top_k * non_local * hidden_dim * 2 * num_layers
    latency_ms = comm / (link_bandwidth_gbps * 1e9 / 8) * 1000
    nodes = [ExpertShard(rank=r, world_size=world_size, total_experts=num_experts).stats()
             for r in range(world_size)]
    return {
        "world_size": world_size,
        "num_experts": num_experts,
        "num_layers": num_layers,
        "experts_per_node": per,
        "remainder_experts": rem,
        "total_memory_gb": round(total_gb, 1),
        "per_node_memory_gb": round(per_gb, 1),
        "memory_savings_pct": round((1 - 1 / world_size) * 100, 1),
        "comm_per_token_bytes": int(comm),
        "comm_latency_ms": round(latency_ms, 3),
        "nodes": nodes,
    }


def balanced_placement(loads, world_size: int) -> list:
    """Expert placement that evens the expected load of the contiguous
    ExpertShard blocks: returns ``order`` with ``order[s]`` = the expert
    stored at position ``s``, so rank ``r`` holds the experts at positions
    ``[r*floor(E/W), ...)`` exactly as ``ExpertShard`` partitions ids.

    ``loads[e]`` is expert e's expected load (e.g. its routing frequency).
    Longest first: experts in decreasing load, each to the rank with the
    least load so far among those whose block still has room (blocks keep
    the ExpertShard sizes; ties go to the lower rank), so the rank holding
    the hottest expert fills up with the coldest ones.  The reference
    partitions by id only (distributed_experts.py:36-80); relabelling experts
    by this order (router columns and expert weights together) leaves the
    model's outputs unchanged and only moves work between ranks.
    """
    E = len(loads)
    W = int(world_size)
    if W <= 1 or E < W:
        return list(range(E))
    per = E // W
    room = [per] * W
    room[-1] += E - per * W
    total = [0.0] * W
    blocks = [[] for _ in range(W)]
    for e in sorted(range(E), key=lambda e: (-float(loads[e]), e)):
        r = min((r for r in range(W) if room[r] > 0), key=lambda r: (total[r], r))
        blocks[r].append(e)
        total[r] += float(loads[e])
        room[r] -= 1
    return [e for b in blocks for e in b]
