"""Routed-expert MoE block on libb200flash: router -> plan -> fused SwiGLU
gather_qmm -> down gather_qmm -> weighted combine.

Mirrors the forward that MLX-Flash patches into mlx-lm MoE blocks
(``mlx_flash_compress/expert_streaming.py:439-472``): softmax gates, top-k,
renormalise, ``switch_mlp`` through ``CachedSwitchLinear`` (``gather_qmm``,
``:224-241``), ``(y * scores[..., None]).sum(-2)``.
"""

import torch

from . import _capi
from ._capi import call, ptr, require_cuda, stream_of
from .mx_compat import MoEPlan, gather_qmv_planned


def route_topk(x: torch.Tensor, wr: torch.Tensor, top_k: int, bias: torch.Tensor = None, renorm: bool = True):
    """``softmax(x @ wr.T + bias)`` top-k -> ``(inds int32 [T,k], scores f32 [T,k])``.

    ``x`` bf16 ``[T, H]``, ``wr`` bf16 ``[E, H]`` (the router weight), ``bias``
    f32 ``[E]`` optional.  Ties go to the lower expert id.
    """
    dev = require_cuda(x, wr, bias)
    if x.dtype != torch.bfloat16 or wr.dtype != torch.bfloat16:
        raise ValueError("route_topk takes bf16 x and router weights")
    T, H = x.shape
    E = wr.shape[0]
    x = _capi.aligned_contiguous(x)
    wr = _capi.aligned_contiguous(wr)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    gates = torch.empty(T, E, dtype=torch.float32, device=dev)
    inds = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    scores = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    call("b2f_moe_route_topk", ptr(x), T, H, ptr(wr), ptr(b), E, top_k, int(renorm), ptr(gates), ptr(inds),
         ptr(scores), stream_of(dev))
    return inds, scores


def switch_glu(x: torch.Tensor, inds: torch.Tensor, gate, up, down, group_size: int = 64, bits: int = 4):
    """SwitchGLU over routed experts: per (token, k) ``down(silu(gate x) * up x)``.

    ``gate``/``up``/``down`` are ``(wq, scales, biases)`` stacked over experts.
    Returns ``[T, k, H]`` bf16 (the layout ``gather_qmm`` gives the reference).
    """
    T, k = inds.shape
    E = gate[0].shape[0]
    K = x.shape[-1]
    tile = 16 if K // group_size <= 32 else 8
    plan = MoEPlan(inds.reshape(-1), E, tile)
    h = gather_qmv_planned(x, plan, *gate, group_size, bits, x_row_div=k, up=up)
    y = gather_qmv_planned(h, plan, *down, group_size, bits)
    return y.reshape(T, k, -1)


def moe_block(x: torch.Tensor, wr: torch.Tensor, gate, up, down, top_k: int, bias=None, renorm=True,
              group_size: int = 64, bits: int = 4, residual: torch.Tensor = None):
    """Full routed MoE block: ``residual + sum_k score_k * expert_k(x)`` (bf16 ``[T, H]``)."""
    inds, scores = route_topk(x, wr, top_k, bias, renorm)
    y = switch_glu(x, inds, gate, up, down, group_size, bits)
    T, H = x.shape
    dev = x.device
    resid = torch.zeros_like(x) if residual is None else residual.contiguous()
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    scratch = torch.empty_like(x)
    # combine through the fused kernel (its RMSNorm output is discarded here)
    call("b2f_combine_rmsnorm", ptr(resid), ptr(y), ptr(scores), T, top_k, ptr(ones), 1e-6, H, ptr(out),
         ptr(scratch), stream_of(dev))
    return out, inds, scores
