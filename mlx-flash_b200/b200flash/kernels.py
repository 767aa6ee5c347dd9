"""Drop-in for ``mlx_flash_compress/kernels/ops.py`` and the Metal shader
``kernels/flash_dequant.metal``: the standalone SwiGLU, the top-k weighted
expert sum and the Q4_0 dequant-GEMV, each one sm_100a kernel.

The reference falls back to plain MLX ops when its Metal kernels are
unavailable; here there is no fallback -- a missing library raises.
"""

import torch

from . import _capi
from ._capi import call, ptr, require_cuda, stream_of

_DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise ValueError(f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` computed in fp32, returned in ``gate``'s dtype (ops.py:48-108)."""
    dev = require_cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError("gate and up must have the same shape and dtype")
    g, u = gate.contiguous(), up.contiguous()
    out = torch.empty_like(g)
    call("b2f_swiglu", ptr(g), ptr(u), ptr(out), g.numel(), _dtype_code(g), stream_of(dev))
    return out


def moe_dispatch(expert_outputs: torch.Tensor, selected_ids: torch.Tensor,
                 routing_weights: torch.Tensor) -> torch.Tensor:
    """Weighted sum of the selected experts' outputs (ops.py:111-135).

    ``expert_outputs`` ``[E, H]``, ``selected_ids`` ``[k]``, ``routing_weights``
    ``[k]`` -> ``[H]``.  A leading token axis on all three (``[T, E, H]``,
    ``[T, k]``, ``[T, k]``) gives ``[T, H]``.
    """
    dev = require_cuda(expert_outputs, selected_ids, routing_weights)
    single = selected_ids.dim() == 1
    eo = expert_outputs.contiguous()
    ids = selected_ids.to(torch.int32).reshape(1 if single else selected_ids.shape[0], -1).contiguous()
    w = routing_weights.to(torch.float32).reshape(ids.shape).contiguous()
    T, k = ids.shape
    E, H = eo.shape[-2], eo.shape[-1]
    stride = 0 if eo.dim() == 2 else E * H
    if eo.dim() == 3 and eo.shape[0] != T:
        raise ValueError("expert_outputs token axis does not match selected_ids")
    out = torch.empty(T, H, dtype=eo.dtype, device=dev)
    call("b2f_moe_dispatch", ptr(eo), stride, E, H, ptr(ids), ptr(w), T, k, _dtype_code(eo), ptr(out),
         stream_of(dev))
    return out[0] if single else out


def flash_dequant_gemv_q4(weights: torch.Tensor, scales: torch.Tensor, x: torch.Tensor,
                          group_size: int = 32) -> torch.Tensor:
    """The ``flash_dequant_gemv_q4`` shader (flash_dequant.metal:19-49): ``y = W_q4 @ x``.

    ``weights`` uint8 ``[M, N/2]`` (low nibble = even column, value
    ``code - 8``), ``scales`` fp16 ``[M, N/group_size]``, ``x`` fp32 ``[N]``
    (or ``[B, N]``) -> fp32 ``[M]`` (or ``[B, M]``).
    """
    dev = require_cuda(weights, scales, x)
    if weights.dtype != torch.uint8 or scales.dtype != torch.float16:
        raise ValueError("weights must be uint8 and scales fp16")
    M = weights.shape[0]
    N = weights.shape[1] * 2
    xs = x.to(torch.float32).reshape(-1, N).contiguous()
    w = _capi.aligned_contiguous(weights)
    y = torch.empty(xs.shape[0], M, dtype=torch.float32, device=dev)
    call("b2f_q4_0_gemv", ptr(w), ptr(scales.contiguous()), ptr(xs), ptr(y), M, N, group_size, xs.shape[0],
         stream_of(dev))
    return y[0] if x.dim() == 1 else y
