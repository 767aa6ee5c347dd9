"""``enable_caching``: the reference's public drop-in for routed-expert models
(``mlx_flash_compress/vllm_integration.py:41-111``), on libb200flash.

A caller that did ``from mlx_flash_compress.vllm_integration import
enable_caching`` swaps that one import.  The model is a PyTorch module tree
shaped like mlx-lm's MoE models (``model.model.layers[i].mlp`` with
``gate``, ``top_k`` and ``switch_mlp.{gate,up,down}_proj`` holding stacked
affine-quantized CUDA weights ``weight``/``scales``/``biases``, optionally
``shared_expert`` and ``shared_expert_gate``).  Every expert stays resident
in HBM, so ``capacity_per_layer`` and ``warmup_task`` only label the state.
"""

from typing import Optional

from .expert_streaming import StreamingState, enable_expert_streaming, enable_skip_fallback, get_warmup_experts


def enable_caching(model, capacity_per_layer: int = 200, model_path: Optional[str] = None,
                   adaptive_skip_threshold: float = 0.0, warmup_task: Optional[str] = None) -> StreamingState:
    """Swap the routed projections for ``CachedSwitchLinear`` and, with
    ``adaptive_skip_threshold > 0``, the MoE forward for the skip-fallback
    forward (LExI); then warm the caches.  Returns the ``StreamingState``."""
    state = enable_expert_streaming(model, capacity_per_layer=capacity_per_layer, model_path=model_path)
    state.skip_threshold = float(adaptive_skip_threshold)
    if adaptive_skip_threshold > 0 and state.caches:
        enable_skip_fallback(model, state.caches, adaptive_skip_threshold=adaptive_skip_threshold)
    if warmup_task and state.caches:
        cache = state.caches[0]
        lists = get_warmup_experts(task=warmup_task, num_layers=len(state.caches), num_experts=cache.num_experts,
                                   top_n=cache.capacity)
        for c, experts in zip(state.caches, lists):
            c.initial_fill(experts)
    else:
        state.warmup()
    return state
