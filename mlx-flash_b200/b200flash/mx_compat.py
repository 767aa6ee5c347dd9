"""MLX quantized-array ops with MLX's signatures, on CUDA torch tensors.

These replace the ``mx.*`` calls the reference makes on its hot path:

* ``quantize``          <- ``mx.quantize`` via ``nn.QuantizedLinear.from_linear``
                           (``mlx_flash_compress/layer_quantization.py:254``)
* ``dequantize``        <- ``mx.dequantize`` (unpack restated at
                           ``mlx_flash_compress/mixed_precision.py:150-171``)
* ``quantized_matmul``  <- the ``nn.QuantizedLinear`` forward
* ``gather_qmm``        <- ``mx.gather_qmm`` in ``CachedSwitchLinear.__call__``
                           (``mlx_flash_compress/expert_streaming.py:230-241``)

Format: affine groups along the last axis; ``wq`` uint32 packed least
significant field first; ``scales``/``biases`` in the weight dtype;
``w = q*scale + bias``.  Every call runs a libb200flash kernel on the tensors'
device; CPU tensors are rejected.
"""

import torch

from . import _capi
from ._capi import DTYPE_CODES, call, ptr, require_cuda, stream_of

SUPPORTED_BITS = (2, 4, 8)
MATMUL_BITS = (4, 8)
GROUP_SIZES = (32, 64, 128)


def _check_format(bits, group_size, allowed=SUPPORTED_BITS):
    if bits not in allowed:
        raise ValueError(f"bits must be one of {allowed}, got {bits}")
    if group_size not in GROUP_SIZES:
        raise ValueError(f"group_size must be one of {GROUP_SIZES}, got {group_size}")


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine", rule: str = "mlx"):
    """Affine-quantize ``w[..., K]`` -> ``(wq uint32[..., K*bits/32], scales, biases)``.

    ``rule="mlx"`` (default): MLX's per-group rule -- the larger-magnitude end
    of the group is the bias and lies exactly on the code grid (the scale is
    negative when that end is the maximum); codes from the f32 scale and bias.
    ``rule="minmax"``: ``scale = (max - min) / (2**bits - 1)``, ``bias = min``
    (the rule stated for the single-linear W[4096, 4096] workload).
    """
    if mode != "affine":
        raise ValueError(f"only mode='affine' is supported, got {mode!r}")
    if rule not in ("mlx", "minmax"):
        raise ValueError(f"rule must be 'mlx' or 'minmax', got {rule!r}")
    _check_format(bits, group_size)
    if w.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported dtype {w.dtype}")
    if w.dim() < 1 or w.shape[-1] % group_size:
        raise ValueError(f"last dimension {tuple(w.shape)[-1:]} must be divisible by group_size {group_size}")
    dev = require_cuda(w)
    K = w.shape[-1]
    lead = tuple(w.shape[:-1])
    rows = w.numel() // K if K else 0
    wc = _capi.aligned_contiguous(w)
    wq = torch.empty(*lead, K * bits // 32, dtype=torch.uint32, device=dev)
    scales = torch.empty(*lead, K // group_size, dtype=w.dtype, device=dev)
    biases = torch.empty_like(scales)
    fn = "b2f_quantize_affine" if rule == "mlx" else "b2f_quantize_affine_minmax"
    call(fn, ptr(wc), DTYPE_CODES[w.dtype], rows, K, bits, group_size, ptr(wq), ptr(scales), ptr(biases),
         stream_of(dev))
    return wq, scales, biases


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4, mode: str = "affine", row_index: torch.Tensor = None) -> torch.Tensor:
    """Inverse of :func:`quantize`; result dtype is the scales' dtype.

    ``row_index`` (int32, optional) gathers rows (embedding lookup).
    """
    if mode != "affine":
        raise ValueError(f"only mode='affine' is supported, got {mode!r}")
    _check_format(bits, group_size)
    if scales.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported scale dtype {scales.dtype}")
    dev = require_cuda(w, scales, biases, row_index)
    K = w.shape[-1] * 32 // bits
    if scales.shape[-1] * group_size != K or biases.shape != scales.shape:
        raise ValueError("scales/biases do not match the packed weight shape")
    w = w.contiguous()
    scales = scales.contiguous()
    biases = biases.contiguous()
    if row_index is not None:
        row_index = row_index.to(torch.int32).contiguous()
        out_lead = tuple(row_index.shape)
    else:
        out_lead = tuple(w.shape[:-1])
    rows = 1
    for d in out_lead:
        rows *= d
    out = torch.empty(*out_lead, K, dtype=scales.dtype, device=dev)
    call("b2f_dequantize_affine", ptr(w), ptr(scales), ptr(biases), DTYPE_CODES[scales.dtype], rows, K,
         bits, group_size, ptr(row_index), ptr(out), stream_of(dev))
    return out


def _sm_count(dev) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


def tc_ksplit(N: int, K: int, sms: int) -> int:
    """K ranges for the tcgen05 GEMM of a decode-sized batch: double the split
    while the 128-row blocks x ranges stay within two CTAs per SM and each
    range keeps at least four 64-wide chunks."""
    blocks = (N + 127) // 128
    chunks = K // 64
    ks = 1
    while blocks * ks * 2 <= 2 * sms and ks * 2 <= chunks // 4:
        ks *= 2
    return ks


def quantized_matmul_engine(M: int, N: int, K: int, bits: int, group_size: int, residual: bool = False) -> str:
    """Kernel ``quantized_matmul`` runs for an ``[M, K] x [N, K]^T`` product:

    * ``"gemv"`` -- the register GEMV (``b2f_qgemv_affine``) for up to 16 rows
      when K has at most 64 groups;
    * ``"tc"`` -- the tcgen05 GEMM (``b2f_qgemm_affine_tcgen05_splitk``) for
      group 64: any K (multiple of 64), K split over the SMs for decode-sized M;
    * ``"gemv_k"`` -- group 32 / 128 with more than 64 groups: the GEMV over K
      ranges of 64 groups, each range adding the previous ones as its residual.
    """
    if group_size == 64 and K % 64 == 0 and (M > 16 or K // group_size > 64 or bits == 8):
        return "tc"
    if K // group_size <= 64:
        return "gemv"
    return "gemv_k"


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4,
                     mode: str = "affine", residual: torch.Tensor = None, engine: str = "auto") -> torch.Tensor:
    """``x @ dequantize(w).T`` for ``x[..., K]`` (bf16) -> ``[..., N]`` bf16.

    ``residual`` (optional, ``[..., N]`` bf16) is added in the same kernel.
    ``engine`` picks the kernel (``quantized_matmul_engine`` for ``"auto"``).
    """
    if not transpose:
        raise ValueError("only transpose=True is supported on this path")
    if mode != "affine":
        raise ValueError(f"only mode='affine' is supported, got {mode!r}")
    _check_format(bits, group_size, MATMUL_BITS)
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16:
        raise ValueError("quantized_matmul takes bf16 activations and bf16 scales/biases")
    dev = require_cuda(x, w, scales, biases, residual)
    N = w.shape[-2]
    K = w.shape[-1] * 32 // bits
    if x.shape[-1] != K:
        raise ValueError(f"x last dim {x.shape[-1]} != K {K}")
    if w.dim() != 2 or tuple(scales.shape) != (N, K // group_size) or biases.shape != scales.shape:
        raise ValueError("w must be [N, K*bits/32] with scales/biases [N, K/group_size]")
    lead = tuple(x.shape[:-1])
    M = x.numel() // K
    if engine == "auto":
        engine = quantized_matmul_engine(M, N, K, bits, group_size, residual is not None)
    if engine not in ("gemv", "tc", "gemv_k"):
        raise ValueError(f"unknown engine {engine!r}")
    if engine == "tc":
        if not tc_supported(K, group_size, bits):
            raise ValueError("the tcgen05 GEMM needs group_size 64 and K % 64 == 0")
        ks = tc_ksplit(N, K, _sm_count(dev)) if M <= 64 else 1
        tile = min(128, max(16, (M + 15) // 16 * 16))
        return quantized_matmul_tc(x, w, scales, biases, group_size, bits, residual, tile=tile, ksplit=ks)
    xc = _capi.aligned_contiguous(x.reshape(M, K))
    out = torch.empty(*lead, N, dtype=torch.bfloat16, device=dev)
    res = None
    if residual is not None:
        res = residual.reshape(M, N).contiguous()
    wc, sc, bc = w.contiguous(), scales.contiguous(), biases.contiguous()
    if engine == "gemv":
        if K // group_size > 64:
            raise ValueError("the register GEMV takes at most 64 groups per row")
        call("b2f_qgemv_affine", ptr(xc), K, M, ptr(wc), ptr(sc), ptr(bc), N, K, bits, group_size, ptr(res),
             ptr(out), N, stream_of(dev))
        return out
    # K ranges of 64 groups: each range's product adds the running sum (bf16)
    kr = 64 * group_size
    out2 = out.reshape(M, N)
    for k0 in range(0, K, kr):
        k1 = min(K, k0 + kr)
        wr = wc[:, k0 * bits // 32: k1 * bits // 32].contiguous()
        sr = sc[:, k0 // group_size: k1 // group_size].contiguous()
        br = bc[:, k0 // group_size: k1 // group_size].contiguous()
        xr = _capi.aligned_contiguous(xc[:, k0:k1])
        prev = res if k0 == 0 else out2.clone()
        call("b2f_qgemv_affine", ptr(xr), k1 - k0, M, ptr(wr), ptr(sr), ptr(br), N, k1 - k0, bits, group_size,
             ptr(prev), ptr(out2), N, stream_of(dev))
    return out


def _moe_tile(K, group_size):
    return 16 if K // group_size <= 32 else 8


def tc_supported(K, group_size, bits):
    """Shapes the tcgen05 grouped GEMM takes (group 64, K % 64 == 0)."""
    return group_size == 64 and K % 64 == 0 and bits in (4, 8)


def quantized_matmul_tc(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                        group_size: int = 64, bits: int = 4, residual: torch.Tensor = None,
                        tile: int = 128, ksplit: int = 1) -> torch.Tensor:
    """``x @ dequantize(w).T`` on the tcgen05 tensor cores (prefill-sized M).

    ``ksplit > 1`` cuts K into ranges whose fp32 partials are summed by a
    second kernel (decode-sized M with few 128-row blocks)."""
    dev = require_cuda(x, w, scales, biases, residual)
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16:
        raise ValueError("bf16 activations and bf16 scales/biases required")
    N = w.shape[-2]
    K = w.shape[-1] * 32 // bits
    if not tc_supported(K, group_size, bits):
        raise ValueError("tcgen05 path needs group_size 64 and K % 64 == 0")
    lead = tuple(x.shape[:-1])
    M = x.numel() // K
    xc = _capi.aligned_contiguous(x.reshape(M, K))
    out = torch.empty(*lead, N, dtype=torch.bfloat16, device=dev)
    res = None if residual is None else residual.reshape(M, N).contiguous()
    if ksplit > 1:
        nb = int(_capi.lib().b2f_qgemm_splitk_workspace_bytes(M, N, int(ksplit)))
        ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=dev)
        call("b2f_qgemm_affine_tcgen05_splitk", ptr(xc), K, M, ptr(w.contiguous()), ptr(scales.contiguous()),
             ptr(biases.contiguous()), N, K, bits, group_size, ptr(res), ptr(out), N, int(tile), int(ksplit),
             ptr(ws), nb, stream_of(dev))
        return out
    call("b2f_qgemm_affine_tcgen05", ptr(xc), K, M, ptr(w.contiguous()), ptr(scales.contiguous()),
         ptr(biases.contiguous()), N, K, bits, group_size, ptr(res), ptr(out), N, int(tile), stream_of(dev))
    return out


def gather_qmm_tc_planned(x_rows: torch.Tensor, plan: "MoEPlan", w, scales, biases, group_size, bits,
                          x_row_index: torch.Tensor = None, x_row_div: int = 1, up=None) -> torch.Tensor:
    """Grouped GEMM over a prepared plan on the tcgen05 tensor cores (plan tile 16..256)."""
    dev = require_cuda(x_rows, w, scales, biases, x_row_index)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    if not tc_supported(K, group_size, bits):
        raise ValueError("tcgen05 path needs group_size 64 and K % 64 == 0")
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    out = torch.empty(plan.A, N, dtype=torch.bfloat16, device=dev)
    wu = su = bu = None
    if up is not None:
        wu, su, bu = (t.contiguous() for t in up)
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_gather_qgemm_affine_tcgen05", ptr(xc), K, ptr(xri), int(x_row_div), plan.A, E, ptr(w.contiguous()),
         ptr(scales.contiguous()), ptr(biases.contiguous()), ptr(wu), ptr(su), ptr(bu), N, K, bits, group_size,
         plan.tile, ptr(plan.workspace), plan.workspace.numel(), ptr(out), N, stream_of(dev))
    return out


def gather_qmm_mma_planned(x_rows: torch.Tensor, plan: "MoEPlan", w, scales, biases, group_size, bits,
                           x_row_index: torch.Tensor = None, x_row_div: int = 1, up=None,
                           x_plan_order: bool = False, out_plan_order: bool = False) -> torch.Tensor:
    """Grouped GEMM over a prepared plan on warp-level tensor-core MMA with the
    4-bit codes unpacked in registers: tile 16 or 32 for decode-sized expert
    tiles (32 unpacks an expert routed 17-32 tokens once instead of twice),
    tile 64 (one matrix) for a dense projection of a whole decode batch.

    ``x_plan_order``: ``x_rows`` is in plan order with permuted columns (the
    ``moe_gather_rows`` layout, or this function's ``out_plan_order`` output).
    ``out_plan_order``: the result keeps that layout (input of the down projection).
    """
    dev = require_cuda(x_rows, w, scales, biases, x_row_index)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    if bits != 4 or group_size != 64 or K % 128 or N % 8 or plan.tile not in (16, 32, 64):
        raise ValueError("the register-unpack MMA path needs 4-bit, group 64, K % 128 == 0, N % 8 == 0, "
                         "tile 16/32/64")
    if plan.tile == 64 and up is not None:
        raise ValueError("64-token tiles take one matrix (no fused up projection)")
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    out = torch.empty(plan.A, N, dtype=torch.bfloat16, device=dev)
    wu = su = bu = None
    if up is not None:
        wu, su, bu = (t.contiguous() for t in up)
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_gather_qgemm_affine_mma", ptr(xc), K, ptr(xri), int(x_row_div), int(x_plan_order), plan.A, E,
         ptr(w.contiguous()), ptr(scales.contiguous()), ptr(biases.contiguous()), ptr(wu), ptr(su), ptr(bu), N, K,
         bits, group_size, plan.tile, ptr(plan.workspace), plan.workspace.numel(), ptr(out), N, int(out_plan_order),
         stream_of(dev))
    return out


def gather_qmm_mma_partials(x_rows: torch.Tensor, plan: "MoEPlan", w, scales, biases, group_size, bits,
                            ksplit: int, x_row_index: torch.Tensor = None, x_row_div: int = 1) -> torch.Tensor:
    """Split-K form of ``gather_qmm_mma_planned`` (plan tile 16 or 64, one
    matrix): fp32 planes ``[n_ranges, A, N]`` whose sum over the first axis is
    the product."""
    dev = require_cuda(x_rows, w, scales, biases, x_row_index)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    lib = _capi.lib()
    nr = int(lib.b2f_mma_splitk_ranges(K, ksplit))
    out = torch.empty(nr, plan.A, N, dtype=torch.float32, device=dev)
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_gather_qgemm_affine_mma_partials", ptr(xc), K, ptr(xri), int(x_row_div), plan.A, E, ptr(w.contiguous()),
         ptr(scales.contiguous()), ptr(biases.contiguous()), N, K, bits, group_size, plan.tile, ptr(plan.workspace),
         plan.workspace.numel(), int(ksplit), ptr(out), out.numel() * 4, stream_of(dev))
    return out


def gather_qmm_2bit_planned(x_rows: torch.Tensor, plan: "MoEPlan", w, scales, biases,
                            x_row_index: torch.Tensor = None, x_row_div: int = 1, up=None) -> torch.Tensor:
    """Grouped GEMM over 2-bit codes (``requantize_4bit_to_2bit`` output: packed
    bytes viewed as uint32 ``[E, N, K/16]``, fp16 or bf16 scales/biases
    ``[E, N, K/64]``) on warp MMA; plan tile 16; ``up`` fuses SwiGLU."""
    dev = require_cuda(x_rows, w, scales, biases, x_row_index)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 16
    if K % 128 or N % 8 or plan.tile != 16:
        raise ValueError("the 2-bit MMA path needs K % 128 == 0, N % 8 == 0 and a plan with tile 16")
    if scales.dtype not in (torch.float16, torch.bfloat16) or biases.dtype != scales.dtype:
        raise ValueError("scales/biases must both be float16 or both bfloat16")
    sdt = 1 if scales.dtype == torch.float16 else 0
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    out = torch.empty(plan.A, N, dtype=torch.bfloat16, device=dev)
    wu = su = bu = None
    if up is not None:
        wu, su, bu = (t.contiguous() for t in up)
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_gather_qgemm_2bit_mma", ptr(xc), K, ptr(xri), int(x_row_div), plan.A, E, ptr(w.contiguous()),
         ptr(scales.contiguous()), ptr(biases.contiguous()), ptr(wu), ptr(su), ptr(bu), N, K, sdt, plan.tile,
         ptr(plan.workspace), plan.workspace.numel(), ptr(out), N, stream_of(dev))
    return out


def moe_gather_rows(x_rows: torch.Tensor, plan: "MoEPlan", x_row_index: torch.Tensor = None,
                    x_row_div: int = 1) -> torch.Tensor:
    """Activation rows in the plan's expert-sorted order (``[A, K]``; rows past
    the planned count are left unwritten), each group of 8 columns in the
    order (0,4,1,5,2,6,3,7) that ``sorted_qmm_tc`` consumes."""
    dev = require_cuda(x_rows, x_row_index)
    K = x_rows.shape[-1]
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    out = torch.empty(plan.A, K, dtype=torch.bfloat16, device=dev)
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_moe_gather_rows", ptr(xc), K, ptr(xri), int(x_row_div), plan.A, plan.E, plan.tile,
         ptr(plan.workspace), plan.workspace.numel(), K, ptr(out), K, stream_of(dev))
    return out


def sorted_qmm_tc(x_sorted: torch.Tensor, plan: "MoEPlan", w, scales, biases, group_size: int, bits: int,
                  up=None, out_sorted: bool = False) -> torch.Tensor:
    """Grouped tcgen05 GEMM over expert-sorted rows (``moe_gather_rows`` layout).

    ``out_sorted=False``: ``out[a] = x[row(a)] . W[e(a)]^T`` for assignment
    ``a`` (natural columns).  ``out_sorted=True``: rows stay in sorted order
    with permuted columns -- the input layout of the next ``sorted_qmm_tc``.
    ``up=(w_up, s_up, b_up)`` fuses the SwitchGLU front half.
    """
    dev = require_cuda(x_sorted, w, scales, biases)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    out = torch.empty(plan.A, N, dtype=torch.bfloat16, device=dev)
    wu = su = bu = None
    if up is not None:
        wu, su, bu = (t.contiguous() for t in up)
    call("b2f_sorted_qgemm_affine_tcgen05", ptr(x_sorted), x_sorted.shape[-1], plan.A, E, ptr(w.contiguous()),
         ptr(scales.contiguous()), ptr(biases.contiguous()), ptr(wu), ptr(su), ptr(bu), N, K, bits, group_size,
         plan.tile, ptr(plan.workspace), plan.workspace.numel(), ptr(out), N, int(out_sorted), stream_of(dev))
    return out


class MoEPlan:
    """Device-side grouping of assignments by expert (output of ``b2f_moe_plan``)."""

    def __init__(self, expert_of: torch.Tensor, num_experts: int, tile: int):
        dev = require_cuda(expert_of)
        self.expert_of = expert_of.to(torch.int32).contiguous().reshape(-1)
        self.A = self.expert_of.numel()
        self.E = int(num_experts)
        self.tile = int(tile)
        nbytes = _capi.lib().b2f_moe_plan_workspace_bytes(self.A, self.E, self.tile)
        self.workspace = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        call("b2f_moe_plan", ptr(self.expert_of), self.A, self.E, self.tile, ptr(self.workspace),
             self.workspace.numel(), ptr(self.status), stream_of(dev))

    def check(self):
        """Synchronising check that every expert id was in range."""
        rc = int(self.status.item())
        if rc:
            raise IndexError("expert index out of range in rhs_indices")


def gather_qmv_planned(x_rows: torch.Tensor, plan: MoEPlan, w, scales, biases, group_size, bits,
                       x_row_index: torch.Tensor = None, x_row_div: int = 1, up=None) -> torch.Tensor:
    """Grouped GEMV over a prepared plan: ``out[a] = x_rows[row(a)] . W[e(a)]^T``.

    ``up=(w_up, s_up, b_up)`` switches to the fused SwitchGLU front half
    ``silu(x.Wg^T) * (x.Wu^T)``.
    """
    dev = require_cuda(x_rows, w, scales, biases, x_row_index)
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    if x_rows.shape[-1] != K:
        raise ValueError(f"x last dim {x_rows.shape[-1]} != K {K}")
    xc = _capi.aligned_contiguous(x_rows.reshape(-1, K))
    out = torch.empty(plan.A, N, dtype=torch.bfloat16, device=dev)
    wu = su = bu = None
    if up is not None:
        wu, su, bu = (t.contiguous() for t in up)
    xri = None if x_row_index is None else x_row_index.to(torch.int32).contiguous()
    call("b2f_gather_qgemv_affine", ptr(xc), K, ptr(xri), int(x_row_div), plan.A, E, ptr(w.contiguous()),
         ptr(scales.contiguous()), ptr(biases.contiguous()), ptr(wu), ptr(su), ptr(bu), N, K, bits,
         group_size, plan.tile, ptr(plan.workspace), plan.workspace.numel(), ptr(out), N, stream_of(dev))
    return out


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               lhs_indices: torch.Tensor = None, rhs_indices: torch.Tensor = None, transpose: bool = True,
               group_size: int = 64, bits: int = 4, mode: str = "affine",
               sorted_indices: bool = False, engine: str = "auto") -> torch.Tensor:
    """``mx.gather_qmm``: per batch element ``x[lhs] @ dequantize(w[rhs]).T``.

    ``x``: ``[..., M, K]`` bf16; ``w``: ``[E, N, K*bits/32]``; result
    ``[*broadcast(batch), M, N]`` bf16.  ``sorted_indices`` is accepted for
    signature compatibility; the kernels always group rows by expert
    themselves.  ``engine`` picks the kernel (``gather_qmm_engine`` for "auto").
    """
    if not transpose:
        raise ValueError("only transpose=True is supported on this path")
    if mode != "affine":
        raise ValueError(f"only mode='affine' is supported, got {mode!r}")
    _check_format(bits, group_size, MATMUL_BITS)
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16:
        raise ValueError("gather_qmm takes bf16 activations and bf16 scales/biases")
    dev = require_cuda(x, w, scales, biases, lhs_indices, rhs_indices)
    if w.dim() != 3:
        raise ValueError("w must be stacked [E, N, K*bits/32]")
    E, N = w.shape[0], w.shape[1]
    K = w.shape[2] * 32 // bits
    if x.dim() < 2 or x.shape[-1] != K:
        raise ValueError(f"x must be [..., M, {K}]")
    M = x.shape[-2]
    xb = tuple(x.shape[:-2])
    nx = 1
    for d in xb:
        nx *= d
    lhs = (torch.arange(nx, device=dev).reshape(xb) if lhs_indices is None else lhs_indices.to(dev).long())
    rhs = (torch.arange(E, device=dev) if rhs_indices is None else rhs_indices.to(dev).long())
    if rhs_indices is None and lhs_indices is None:
        rhs = rhs.reshape(E, *([1] * 0))
    lhs_b, rhs_b = torch.broadcast_tensors(lhs, rhs)
    batch = tuple(lhs_b.shape)
    lhs_f = lhs_b.reshape(-1)
    rhs_f = rhs_b.reshape(-1)
    # assignment a = (batch element, m): x row = lhs*M + m, expert = rhs
    m_idx = torch.arange(M, device=dev)
    x_row = (lhs_f[:, None] * M + m_idx[None, :]).reshape(-1).to(torch.int32)
    expert_of = rhs_f[:, None].expand(-1, M).reshape(-1).to(torch.int32)
    A = expert_of.numel()
    if engine == "auto":
        engine = gather_qmm_engine(A, E, N, K, bits, group_size)
    x2 = x.reshape(nx * M, K)
    if engine == "mma":
        plan = MoEPlan(expert_of, E, 16)
        out = gather_qmm_mma_planned(x2, plan, w, scales, biases, group_size, bits, x_row_index=x_row)
    elif engine == "tc_sorted":
        plan = MoEPlan(expert_of, E, 64 if A >= 64 * E else 32)
        xs = moe_gather_rows(x2, plan, x_row_index=x_row)
        out = sorted_qmm_tc(xs, plan, w, scales, biases, group_size, bits)
    elif engine == "tc":
        plan = MoEPlan(expert_of, E, 32)
        out = gather_qmm_tc_planned(x2, plan, w, scales, biases, group_size, bits, x_row_index=x_row)
    elif engine == "gemv":
        if K // group_size > 64:
            raise ValueError("the register GEMV takes at most 64 groups per row; use group_size 64")
        plan = MoEPlan(expert_of, E, _moe_tile(K, group_size))
        out = gather_qmv_planned(x2, plan, w, scales, biases, group_size, bits, x_row_index=x_row)
    else:
        raise ValueError(f"unknown engine {engine!r}")
    return out.reshape(*batch, M, N)


def gather_qmm_engine(A: int, E: int, N: int, K: int, bits: int, group_size: int) -> str:
    """Kernel ``gather_qmm`` runs for ``A`` (token, expert) assignments over
    ``E`` stacked ``[N, K]`` experts:

    * ``"mma"`` -- warp-level MMA with the 4-bit codes unpacked in registers
      (``b2f_gather_qgemm_affine_mma``) while experts average at most 32
      assignments (decode): 4-bit, group 64, K % 128 == 0, N % 8 == 0;
    * ``"tc_sorted"`` -- rows gathered into expert order, then the tcgen05
      grouped GEMM (``b2f_sorted_qgemm_affine_tcgen05``) for prefill-sized
      batches: group 64 with an even group count;
    * ``"tc"`` -- the per-slot tcgen05 GEMM for other group-64 shapes;
    * ``"gemv"`` -- the register GEMV (group 32 / 128, at most 64 groups).
    """
    if bits == 4 and group_size == 64 and K % 128 == 0 and N % 8 == 0 and A <= 32 * E:
        return "mma"
    if group_size == 64 and K % 64 == 0:
        return "tc_sorted" if (K // 64) % 2 == 0 else "tc"
    return "gemv"
