"""Routed-expert MoE block on libb200flash: router -> plan -> fused SwiGLU
gather_qmm -> down gather_qmm -> weighted combine.

Mirrors the forward that MLX-Flash patches into mlx-lm MoE blocks
(``mlx_flash_compress/expert_streaming.py:439-472``): softmax gates, top-k,
the LExI skip mask, renormalise, ``switch_mlp`` through ``CachedSwitchLinear``
(``gather_qmm``, ``:224-241``), ``(y * scores[..., None]).sum(-2)``, plus the
gated shared expert.
"""

import torch

from . import _capi
from ._capi import call, ptr, require_cuda, stream_of
from .mx_compat import (MoEPlan, gather_qmm_engine, gather_qmm_mma_planned, gather_qmm_tc_planned,
                        gather_qmv_planned, moe_gather_rows, sorted_qmm_tc)

GATINGS = {"softmax": 0, "sigmoid": 1}


def route_topk(x: torch.Tensor, wr: torch.Tensor, top_k: int, bias: torch.Tensor = None, renorm: bool = True,
               gating: str = "softmax", skip_threshold: float = 0.0):
    """Top-k routing -> ``(inds int32 [T,k], scores f32 [T,k])``.

    ``gating="softmax"``: gates ``softmax(x @ wr.T + bias)`` (the reference,
    ``expert_streaming.py:440``); ``"sigmoid"``: ``sigmoid`` per expert.
    ``skip_threshold > 0`` applies the LExI mask of the skip-fallback forward
    (``expert_streaming.py:451-457``): slot j >= 1 gets score 0 where the top
    gate exceeds ``skip_threshold`` times it.  ``renorm`` then divides the
    scores by their sum when it is positive.  ``x`` bf16 ``[T, H]``, ``wr``
    bf16 ``[E, H]``, ``bias`` f32 ``[E]`` optional.  Slots are in descending
    gate order; ties go to the lower expert id.
    """
    dev = require_cuda(x, wr, bias)
    if x.dtype != torch.bfloat16 or wr.dtype != torch.bfloat16:
        raise ValueError("route_topk takes bf16 x and router weights")
    if gating not in GATINGS:
        raise ValueError(f"gating must be one of {tuple(GATINGS)}, got {gating!r}")
    if skip_threshold < 0:
        raise ValueError("skip_threshold must be >= 0")
    T, H = x.shape
    E = wr.shape[0]
    x = _capi.aligned_contiguous(x)
    wr = _capi.aligned_contiguous(wr)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    gates = torch.empty(T, E, dtype=torch.float32, device=dev)
    inds = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    scores = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    call("b2f_moe_route_topk_ex", ptr(x), T, H, ptr(wr), ptr(b), E, top_k, int(renorm), GATINGS[gating],
         float(skip_threshold), ptr(gates), ptr(inds), ptr(scores), stream_of(dev))
    return inds, scores


def shared_gate(x: torch.Tensor, w_gate: torch.Tensor) -> torch.Tensor:
    """``sigmoid(x @ w_gate.T)`` f32 ``[T, 1]`` (``shared_expert_gate``, expert_streaming.py:468-469)."""
    dev = require_cuda(x, w_gate)
    T, H = x.shape
    w = _capi.aligned_contiguous(w_gate.reshape(1, H).to(torch.bfloat16))
    out = torch.empty(T, 1, dtype=torch.float32, device=dev)
    call("b2f_router_logits", ptr(_capi.aligned_contiguous(x)), T, H, ptr(w), None, 1, 1, ptr(out), stream_of(dev))
    return out


def switch_glu(x: torch.Tensor, inds: torch.Tensor, gate, up, down, group_size: int = 64, bits: int = 4,
               engine: str = "auto"):
    """SwitchGLU over routed experts: per (token, k) ``down(silu(gate x) * up x)``.

    ``gate``/``up``/``down`` are ``(wq, scales, biases)`` stacked over experts.
    Returns ``[T, k, H]`` bf16 (the layout ``gather_qmm`` gives the reference).
    The kernels follow ``gather_qmm_engine``: warp MMA at decode density (the
    SwiGLU rows stay in plan order between the two GEMMs), the row gather +
    sorted tcgen05 GEMMs at prefill density, else tcgen05 or the GEMV.
    """
    T, k = inds.shape
    E, I = gate[0].shape[0], gate[0].shape[1]
    K = x.shape[-1]
    A = T * k
    if engine == "auto":
        engine = gather_qmm_engine(A, E, I, K, bits, group_size)
        if engine == "mma" and (I % 128 or (K // group_size) % 2):
            engine = "tc" if group_size == 64 else "gemv"
        if engine == "tc_sorted" and (I // 64) % 2:
            engine = "tc"
    if engine == "mma":
        plan = MoEPlan(inds.reshape(-1), E, 16)
        h = gather_qmm_mma_planned(x, plan, *gate, group_size, bits, x_row_div=k, up=up, out_plan_order=True)
        y = gather_qmm_mma_planned(h, plan, *down, group_size, bits, x_plan_order=True)
    elif engine == "tc_sorted":
        plan = MoEPlan(inds.reshape(-1), E, 64 if A >= 64 * E else 32)
        xs = moe_gather_rows(x, plan, x_row_div=k)
        h = sorted_qmm_tc(xs, plan, *gate, group_size, bits, up=up, out_sorted=True)
        y = sorted_qmm_tc(h, plan, *down, group_size, bits)
    elif engine == "tc":
        plan = MoEPlan(inds.reshape(-1), E, 32)
        h = gather_qmm_tc_planned(x, plan, *gate, group_size, bits, x_row_div=k, up=up)
        y = gather_qmm_tc_planned(h, plan, *down, group_size, bits)
    elif engine == "gemv":
        plan = MoEPlan(inds.reshape(-1), E, 16 if K // group_size <= 32 else 8)
        h = gather_qmv_planned(x, plan, *gate, group_size, bits, x_row_div=k, up=up)
        y = gather_qmv_planned(h, plan, *down, group_size, bits)
    else:
        raise ValueError(f"unknown engine {engine!r}")
    return y.reshape(T, k, -1)


def combine(y: torch.Tensor, scores: torch.Tensor, residual: torch.Tensor = None) -> torch.Tensor:
    """``residual + sum_k scores[:, k] * y[:, k]`` (bf16 ``[T, H]``) from ``y``
    bf16 ``[T, k, H]`` and f32 ``scores [T, k]`` (``kernels/ops.py:111-135``)."""
    T, k, H = y.shape
    dev = y.device
    resid = torch.zeros(T, H, dtype=torch.bfloat16, device=dev) if residual is None else residual.contiguous()
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    scratch = torch.empty_like(out)
    call("b2f_combine_rmsnorm", ptr(resid), ptr(y.contiguous()), ptr(scores.to(torch.float32).contiguous()), T, k,
         ptr(ones), 1e-6, H, ptr(out), ptr(scratch), stream_of(dev))
    return out


def _stack1(t):
    wq, sc, bi = t
    return (wq if wq.dim() == 3 else wq.unsqueeze(0), sc if sc.dim() == 3 else sc.unsqueeze(0),
            bi if bi.dim() == 3 else bi.unsqueeze(0))


def moe_block(x: torch.Tensor, wr: torch.Tensor, gate, up, down, top_k: int, bias=None, renorm=True,
              group_size: int = 64, bits: int = 4, residual: torch.Tensor = None, gating: str = "softmax",
              skip_threshold: float = 0.0, shared=None, engine: str = "auto"):
    """Full MoE block: ``residual + sum_k score_k * expert_k(x)`` (bf16 ``[T, H]``)
    plus, with ``shared=(gate, up, down, gate_weight)``, the shared expert
    ``sigmoid(x . gate_weight) * shared_mlp(x)`` (expert_streaming.py:466-470;
    ``gate_weight`` bf16 ``[1, H]`` or None for an ungated shared expert, the
    projections ``(wq, scales, biases)`` of one dense SwiGLU MLP)."""
    inds, scores = route_topk(x, wr, top_k, bias, renorm, gating, skip_threshold)
    y = switch_glu(x, inds, gate, up, down, group_size, bits, engine)
    T, H = x.shape
    dev = x.device
    resid = torch.zeros_like(x) if residual is None else residual.contiguous()
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    scratch = torch.empty_like(x)
    st = stream_of(dev)
    # combine through the fused kernel (its RMSNorm output is discarded here)
    call("b2f_combine_rmsnorm", ptr(resid), ptr(y), ptr(scores), T, top_k, ptr(ones), 1e-6, H, ptr(out),
         ptr(scratch), st)
    if shared is not None:
        sg, su, sd, sw = shared
        ys = switch_glu(x, torch.zeros(T, 1, dtype=torch.int32, device=dev), _stack1(sg), _stack1(su), _stack1(sd),
                        group_size, bits, engine).reshape(T, H)
        g = shared_gate(x, sw) if sw is not None else torch.ones(T, 1, dtype=torch.float32, device=dev)
        call("b2f_combine_rmsnorm", ptr(out), ptr(ys), ptr(g), T, 1, ptr(ones), 1e-6, H, ptr(out), ptr(scratch), st)
    return out, inds, scores
