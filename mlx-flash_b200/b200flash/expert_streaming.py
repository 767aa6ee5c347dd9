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

from dataclasses import dataclass, field

import torch

from . import mx_compat


class ResidentExpertCache:
    """Stacked per-projection expert weights with the reference cache's fields
    (``weights``, ``scales``, ``biases`` keyed by projection name, ``lookup``
    int32 [num_experts], ``hit_mask``, ``_indices_buffer``) and its
    ``ExpertCache`` methods (``initial_fill``, ``update_between_tokens``,
    ``stats``; ``expert_streaming.py:247-360``).  Every expert stays
    resident: ``capacity`` is recorded, the hit mask is all ones, and no
    expert is ever evicted or loaded between tokens."""

    def __init__(self, weights: dict, scales: dict, biases: dict, num_experts: int, expert_ids=None, device=None,
                 layer_idx: int = 0, capacity: int = None):
        dev = device or next(iter(weights.values())).device
        self.weights, self.scales, self.biases = weights, scales, biases
        self.num_experts = int(num_experts)
        self.layer_idx = int(layer_idx)
        self.capacity = self.num_experts if capacity is None else min(int(capacity), self.num_experts)
        ids = list(range(self.num_experts)) if expert_ids is None else [int(e) for e in expert_ids]
        self.cached_ids = ids
        lookup = torch.zeros(self.num_experts, dtype=torch.int32)
        hit = torch.zeros(self.num_experts, dtype=torch.float32)
        for slot, eid in enumerate(ids):
            lookup[eid] = slot
            hit[eid] = 1.0
        self.lookup = lookup.to(dev)
        self.hit_mask = hit.to(dev)
        self.identity = ids == list(range(self.num_experts))
        self._indices_buffer = []
        self.total_tokens = 0
        self.cache_updates = 0

    def initial_fill(self, expert_ids=None):
        """Nothing to load: the stacked weights already hold every expert."""

    def update_between_tokens(self):
        """Drop the recorded routing (every routed expert is resident: no misses)."""
        if self._indices_buffer:
            self._indices_buffer.clear()
            self.total_tokens += 1

    def stats(self):
        return {"layer": self.layer_idx, "cached": len(self.cached_ids), "capacity": self.capacity,
                "coverage": len(self.cached_ids) / max(self.num_experts, 1), "tokens": self.total_tokens,
                "updates": self.cache_updates}


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


@dataclass
class StreamingState:
    """The reference's ``StreamingState`` (``expert_streaming.py:363-397``)."""

    caches: list = field(default_factory=list)
    st_map: object = None
    model: object = None
    skip_threshold: float = 0.0

    def warmup(self):
        for cache in self.caches:
            cache.initial_fill()
        if self.caches:
            torch.cuda.synchronize(self.caches[0].lookup.device)

    def update(self):
        for cache in self.caches:
            cache.update_between_tokens()

    def stats(self):
        return [c.stats() for c in self.caches]

    def total_cached(self):
        return sum(len(c.cached_ids) for c in self.caches)

    def avg_coverage(self):
        if not self.caches:
            return 0
        return sum(c.stats()["coverage"] for c in self.caches) / len(self.caches)

    def cleanup(self):
        if self.st_map:
            self.st_map.close()


_PROJS = ("gate_proj", "up_proj", "down_proj")


def _model_layers(model):
    if hasattr(model, "model") and hasattr(model.model, "layers"):
        return model.model.layers
    if hasattr(model, "layers"):
        return model.layers
    return None


def _switch_of(mlp):
    switch = getattr(mlp, "switch_mlp", None)
    if switch is None:
        bsm = getattr(mlp, "block_sparse_moe", None)
        if bsm is not None:
            switch = getattr(bsm, "switch_mlp", None)
    return switch


def enable_expert_streaming(model, capacity_per_layer=200, model_path=None):
    """Swap every layer's routed projections (``mlp.switch_mlp.{gate,up,down}_proj``,
    or Mixtral's ``block_sparse_moe.switch_mlp``) for ``CachedSwitchLinear``
    over a ``ResidentExpertCache`` of their stacked CUDA weights
    (``expert_streaming.py:510-603``).  ``model_path`` opens the model's
    safetensors (``expert_loader.SafetensorsMap``) only for weights a
    projection does not already hold."""
    layers = _model_layers(model)
    if layers is None:
        raise ValueError("Cannot find model layers")
    state = StreamingState(model=model)
    if model_path:
        from .expert_loader import SafetensorsMap, find_shards

        state.st_map = SafetensorsMap(find_shards(model_path))
    for layer_idx, layer in enumerate(layers):
        mlp = getattr(layer, "mlp", None)
        if mlp is None:
            continue
        switch = _switch_of(mlp)
        if switch is None:
            continue
        mods = {p: getattr(switch, p, None) for p in _PROJS}
        mods = {p: m for p, m in mods.items() if m is not None and getattr(m, "weight", None) is not None
                and m.weight.dim() == 3}
        if not mods:
            continue
        num_experts = next(iter(mods.values())).weight.shape[0]
        cache = ResidentExpertCache({p: m.weight for p, m in mods.items()}, {p: m.scales for p, m in mods.items()},
                                    {p: m.biases for p, m in mods.items()}, num_experts, layer_idx=layer_idx,
                                    capacity=capacity_per_layer)
        state.caches.append(cache)
        for p, m in mods.items():
            setattr(switch, p, CachedSwitchLinear(cache, p, getattr(m, "group_size", 64), getattr(m, "bits", 4),
                                                  getattr(m, "mode", "affine")))
    return state


def _qlinear(m):
    return (m.weight, m.scales, m.biases)


def enable_skip_fallback(model, caches: list, adaptive_skip_threshold: float = 0.0):
    """Replace each cached layer's MoE forward with the reference's skip-fallback
    forward (``expert_streaming.py:402-479``) on libb200flash kernels: softmax
    router + top-k + LExI mask + renormalisation in one kernel
    (``b2f_moe_route_topk_ex``), the routed SwiGLU experts
    (``moe.switch_glu``), the weighted combine, and ``shared_expert`` gated by
    ``sigmoid(shared_expert_gate(x))`` when the block has them."""
    import types

    from . import moe

    layers = _model_layers(model)
    if layers is None:
        return
    by_layer = {c.layer_idx: c for c in caches}
    thr = float(adaptive_skip_threshold)
    for layer_idx, layer in enumerate(layers):
        if layer_idx not in by_layer or not hasattr(layer, "mlp"):
            continue
        cache = by_layer[layer_idx]
        mlp = layer.mlp
        switch = _switch_of(mlp)
        gs = switch.gate_proj.group_size
        bits = switch.gate_proj.bits

        def patched_forward(self, x, cache=cache, switch=switch, gs=gs, bits=bits):
            shape = x.shape
            x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
            T, H = x2.shape
            inds, scores = moe.route_topk(x2, self.gate.weight.to(torch.bfloat16), self.top_k, None, True,
                                          "softmax", thr)
            cache._indices_buffer.append(inds)
            local = inds if cache.identity else cache.lookup[inds.long()].to(torch.int32)
            w = {p: (cache.weights[p], cache.scales[p], cache.biases[p]) for p in _PROJS}
            y = moe.switch_glu(x2, local, w["gate_proj"], w["up_proj"], w["down_proj"], gs, bits)
            out = moe.combine(y, scores)
            se = getattr(self, "shared_expert", None)
            if se is not None:
                sg = getattr(self, "shared_expert_gate", None)
                shared = tuple(_qlinear(getattr(se, p)) for p in _PROJS)
                ys = moe.switch_glu(x2, torch.zeros(T, 1, dtype=torch.int32, device=x2.device),
                                    *(moe._stack1(t) for t in shared), gs, bits).reshape(T, H)
                g = (moe.shared_gate(x2, sg.weight.to(torch.bfloat16)) if sg is not None
                     else torch.ones(T, 1, dtype=torch.float32, device=x2.device))
                out = moe.combine(ys.reshape(T, 1, H), g, residual=out)
            return out.reshape(shape)

        mlp.forward = types.MethodType(patched_forward, mlp)


def get_warmup_experts(task: str = "general", num_layers: int = 24, num_experts: int = 60, top_n: int = 30) -> list:
    """Hot experts per layer for a task (the reference falls back to the first
    ``top_n``; with every expert resident the list only labels the warm-up)."""
    return [list(range(min(top_n, num_experts))) for _ in range(num_layers)]
