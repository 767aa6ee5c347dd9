"""``CachedSwitchLinear`` of ``mlx_flash_compress/expert_streaming.py:213-241``
for HBM-resident experts.

The reference swaps this module in for MLX's ``QuantizedSwitchLinear``: the
routed expert ids are remapped through the cache's lookup table (global id ->
slot of the stacked, cached expert weights) and the projection runs as
``mx.gather_qmm``.  On a 180 GB B200 every expert of the layer (or of this
rank's ``ExpertShard``) stays resident, so the cache here is the stacked
weights plus a lookup table (identity, or global id -> local slot for an
expert-parallel shard); the SSD streaming / LCP eviction machinery around it
is not part of this path.
"""

import torch

from . import mx_compat


class ResidentExpertCache:
    """Stacked per-projection expert weights with the reference cache's fields
    (``weights``, ``scales``, ``biases`` keyed by projection name, ``lookup``
    int32 [num_experts], ``hit_mask``, ``_indices_buffer``)."""

    def __init__(self, weights: dict, scales: dict, biases: dict, num_experts: int, expert_ids=None, device=None):
        dev = device or next(iter(weights.values())).device
        self.weights, self.scales, self.biases = weights, scales, biases
        self.num_experts = int(num_experts)
        ids = list(range(self.num_experts)) if expert_ids is None else [int(e) for e in expert_ids]
        self.cached_ids = ids
        lookup = torch.zeros(self.num_experts, dtype=torch.int32)
        hit = torch.zeros(self.num_experts, dtype=torch.float32)
        for slot, eid in enumerate(ids):
            lookup[eid] = slot
            hit[eid] = 1.0
        self.lookup = lookup.to(dev)
        self.hit_mask = hit.to(dev)
        self._indices_buffer = []


class CachedSwitchLinear(torch.nn.Module):
    """Drop-in for the reference module: ``forward(x, indices, sorted_indices=False)``."""

    def __init__(self, cache, proj_name: str, group_size: int, bits: int, mode: str = "affine"):
        super().__init__()
        self._cache = cache
        self._proj_name = proj_name
        self.group_size = group_size
        self.bits = bits
        self.mode = "affine" if mode in (0, "affine") else mode

    def forward(self, x, indices, sorted_indices: bool = False):
        if self._proj_name == "gate_proj":
            self._cache._indices_buffer.append(indices)
        local = self._cache.lookup[indices.long()]
        return mx_compat.gather_qmm(x, self._cache.weights[self._proj_name], self._cache.scales[self._proj_name],
                                    self._cache.biases.get(self._proj_name), rhs_indices=local, transpose=True,
                                    group_size=self.group_size, bits=self.bits, mode=self.mode,
                                    sorted_indices=sorted_indices)
