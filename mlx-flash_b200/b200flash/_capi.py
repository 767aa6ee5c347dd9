"""ctypes binding of libb200flash.so (the C ABI declared in include/b2f.h).

This is the only place the package touches the shared library.  There is no
CPU or framework fallback: if the library is missing or no CUDA device is
present, every compute entry point raises.
"""

import contextlib
import ctypes
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libb200flash.so")

B2F_OK = 0
B2F_ERR_INVALID = -1
B2F_ERR_UNSUPPORTED = -2
B2F_ERR_ALIGN = -3
B2F_ERR_CUDA = -4
B2F_ERR_TIMEOUT = -5
B2F_ERR_WORKSPACE = -6

DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/b2f.h
SIGNATURES = {
    "b2f_version": (ctypes.c_char_p, []),
    "b2f_status_string": (ctypes.c_char_p, [_I]),
    "b2f_last_error_string": (ctypes.c_char_p, []),
    "b2f_quantize_affine": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "b2f_quantize_affine_minmax": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "b2f_dequantize_affine": (_I, [_P, _P, _P, _I, _I64, _I64, _I, _I, _P, _P, _P]),
    "b2f_qgemv_affine": (_I, [_P, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I, _P, _P, _I64, _P]),
    "b2f_moe_plan_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "b2f_moe_plan_max_slots": (_I64, [_I64, _I64, _I]),
    "b2f_moe_plan": (_I, [_P, _I64, _I64, _I, _P, _I64, _P, _P]),
    "b2f_ep_plan": (_I, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P,
                         _I64, _P, _P]),
    "b2f_ep_combine_partial": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _P]),
    "b2f_qgemm_splitk_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "b2f_qgemm_affine_tcgen05_splitk": (_I, [_P, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I, _P, _P, _I64, _I, _I, _P,
                                             _I64, _P]),
    "b2f_qgemm_splitk_ranges": (_I, [_I64, _I]),
    "b2f_qgemm_affine_tcgen05_partials": (_I, [_P, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I, _I, _I, _P, _I64,
                                               _P]),
    "b2f_combine_rmsnorm_partials": (_I, [_P, _P, _I, _I64, _P, _F, _I64, _P, _P, _P]),
    "b2f_qk_norm_rope_kv_append_partials": (_I, [_P, _I, _I64, _I64, _I64, _I64, _P, _P, _F, _F, _P, _P, _P, _P,
                                                 _P, _P, _P, _I64, _I64, _I, _P]),
    "b2f_moe_route_plan": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I, _P, _P, _P, _I, _P, _I64, _P, _P]),
    "b2f_gather_qgemm_affine_mma": (_I, [_P, _I64, _P, _I64, _I, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64,
                                         _I, _I, _I, _P, _I64, _P, _I64, _I, _P]),
    "b2f_mma_splitk_ranges": (_I, [_I64, _I]),
    "b2f_mma_splitk_workspace_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "b2f_gather_qgemm_affine_mma_partials": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I,
                                                  _I, _P, _I64, _I, _P, _I64, _P]),
    "b2f_gather_qgemm_2bit_mma": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I,
                                       _P, _I64, _P, _I64, _P]),
    "b2f_moe_gather_rows": (_I, [_P, _I64, _P, _I64, _I64, _I64, _I, _P, _I64, _I64, _P, _I64, _P]),
    "b2f_sorted_qgemm_affine_tcgen05": (_I, [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64, _I64, _I, _I, _I,
                                             _P, _I64, _P, _I64, _I, _P]),
    "b2f_attn_row_head_mean": (_I, [_P, _I, _I64, _I64, _I64, _I, ctypes.c_float, _P, _P, _P]),
    "b2f_qkv_head_mean_probs_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "b2f_qkv_head_mean_probs": (_I, [_P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I,
                                     _I, ctypes.c_float, _I, _P, _I64, _P, _I64, _I, ctypes.c_float, _P]),
    "b2f_evict_keep_indices": (_I, [_P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "b2f_kv_pages_gather": (_I, [_P, _P, _P, _P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                 _I64, _I, _P]),
    "b2f_gather_tokens": (_I, [_P, _P, _I64, _I64, _I64, _P, _I64, _P]),
    "b2f_q4_0_gemv": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _I64, _P]),
    "b2f_swiglu": (_I, [_P, _P, _P, _I64, _I, _P]),
    "b2f_moe_dispatch": (_I, [_P, _I64, _I64, _I64, _P, _P, _I64, _I64, _I, _P, _P]),
    "b2f_requant_4to2": (_I, [_P, _I64, _I64, _P, _P, _I, _I64, _P, _P, _P, _P]),
    "b2f_dequant_2bit": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _P]),
    "b2f_fake_quant_sym": (_I, [_P, _I, _I64, _I, _P, _P, _P]),
    "b2f_gather_qgemv_affine": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64,
                                     _I64, _I, _I, _I, _P, _I64, _P, _I64, _P]),
    "b2f_qgemm_affine_tcgen05": (_I, [_P, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I, _P, _P, _I64, _I, _P]),
    "b2f_gather_qgemm_affine_tcgen05": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _I64,
                                             _I64, _I, _I, _I, _P, _I64, _P, _I64, _P]),
    "b2f_kv_packed_len": (_I64, [_I64, _I, _I]),
    "b2f_kv_num_groups": (_I64, [_I64, _I]),
    "b2f_kv_quantize_sym": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _I64, _P, _P, _I64, _P]),
    "b2f_kv_dequantize_sym": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _I, _I, _P, _P]),
    "b2f_qkv_decode_attn_workspace_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "b2f_qkv_decode_attn": (_I, [_P, _P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                 _I64, _I, _I, _F, _I, _P, _I64, _P, _P]),
    "b2f_qkv_decode_attn_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                         _I64, _I, _I, _F, _I, _P, _P]),
    "b2f_combine_rmsnorm": (_I, [_P, _P, _P, _I64, _I64, _P, _F, _I64, _P, _P, _P]),
    "b2f_qk_norm_rope_kv_append": (_I, [_P, _I64, _I64, _I64, _I64, _P, _P, _F, _F, _P, _P, _P, _P, _P, _P,
                                        _P, _I64, _I64, _I, _P]),
    "b2f_moe_route_topk": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I, _P, _P, _P, _P]),
    "b2f_moe_route_topk_ex": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I, _I, _F, _P, _P, _P, _P]),
    "b2f_moe_route_plan_ex": (_I, [_P, _I64, _I64, _P, _P, _I64, _I64, _I, _I, _F, _P, _P, _P, _I, _P, _I64, _P,
                                   _P]),
    "b2f_router_logits": (_I, [_P, _I64, _I64, _P, _P, _I64, _I, _P, _P]),
    "b2f_device_status": (_I, [_P, _I]),
    "b2f_set_wait_limit_ns": (_I, [_I64]),
    "b2f_set_producer_stall": (_I, [_I]),
    "b2f_set_launch_pdl": (_I, [_I]),
    "b2f_mma_packed_bytes": (_I64, [_I64, _I64, _I64, _I]),
    "b2f_mma_repack": (_I, [_P, _P, _P, _I64, _I64, _I64, _I, _P, _I64, _P]),
    "b2f_gather_qgemm_affine_mma_packed": (_I, [_P, _I64, _P, _I64, _I, _I64, _I64, _P, _P, _I64, _I64, _I, _I, _I,
                                                _P, _I64, _P, _I64, _I, _P, _I64, _I, _P]),
    "b2f_mma_streamk_workspace_bytes": (_I64, []),
    "b2f_qgemm_decode_planes": (_I, [_I64, _I64, _I64]),
    "b2f_qgemm_affine_decode_partials": (_I, [_P, _I64, _I64, _P, _P, _P, _I64, _I64, _I, _I, _P, _I64, _P]),
    "b2f_ipc_export": (_I, [_P, _P, _P]),
    "b2f_ipc_import": (_I, [_P, _P]),
    "b2f_ipc_close": (_I, [_P]),
    "b2f_ep_p2p_region_bytes": (_I64, [_I64, _I64, _I64, _I64, _P, _P]),
    "b2f_ep_p2p_dispatch": (_I, [_P, _I64, _P, _I64, _I64, _I, _I, _P, _I64, _I64, _I64, _P, _P, _P, _P]),
    "b2f_ep_p2p_wait": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "b2f_ep_p2p_plan": (_I, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _I, _I64, _I64, _I64, _I64, _I64, _I, _P, _P,
                             _P, _P, _I64, _P, _P, _P, _P]),
    "b2f_ep_p2p_combine_rmsnorm": (_I, [_P, _P, _I64, _I64, _P, _I64, _I, _P, _F, _I64, _P, _P, _P, _P, _P]),
    "b2f_ep_p2p_combine": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _I, _I, _P, _P]),
    "b2f_ep_a2a_row_pitch": (_I64, [_I64, _I64]),
    "b2f_ep_a2a_dispatch": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _P, _P]),
    "b2f_ep_a2a_plan": (_I, [_P, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P, _I64, _P, _P]),
    "b2f_ep_a2a_combine": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _I64, _P]),
    "b2f_argmax_rows": (_I, [_P, _I64, _I64, _P, _P]),
}

_lib = None


class B2FError(RuntimeError):
    """A libb200flash call failed on the device side (CUDA error, timeout, workspace)."""


def lib():
    """Load libb200flash.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libb200flash.so not found at {LIB_PATH}; build it with "
                "`python mlx-flash_b200/b200flash/_build.py` (nvcc, sm_100a)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_text(rc: int) -> str:
    return lib().b2f_status_string(rc).decode()


def check(rc: int, what: str) -> None:
    """Turn a B2F status into the exception the reference API would raise."""
    if rc == B2F_OK:
        return
    msg = f"{what}: {status_text(rc)}"
    if rc == B2F_ERR_CUDA:
        msg += f" ({lib().b2f_last_error_string().decode()})"
    if rc in (B2F_ERR_INVALID, B2F_ERR_UNSUPPORTED, B2F_ERR_ALIGN):
        raise ValueError(msg)
    raise B2FError(msg)


def call(name: str, *args) -> int:
    """Invoke an entry point and raise on a non-zero status."""
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc


def require_cuda(*tensors) -> torch.device:
    """All tensors must live on one CUDA device; returns it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("b200flash kernels take CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor arguments")
    return dev


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def device_status(clear: bool = True) -> int:
    """The library's sticky device status (0, or B2F_ERR_TIMEOUT after a
    bounded wait gave up); synchronises the device."""
    st = ctypes.c_int32(0)
    rc = lib().b2f_device_status(ctypes.byref(st), int(clear))
    if rc != 0:
        raise RuntimeError(f"b2f_device_status failed: {rc}")
    return int(st.value)


@contextlib.contextmanager
def dependent_launches(on: bool = True):
    """Launch this thread's library kernels as programmatic dependent
    launches inside the block (each may be scheduled while its predecessor in
    the stream finishes; results are unchanged); a CUDA graph captured inside
    keeps the dependent edges."""
    prev = int(lib().b2f_set_launch_pdl(int(bool(on))))
    try:
        yield
    finally:
        lib().b2f_set_launch_pdl(prev)


def stream_of(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def aligned_contiguous(t: torch.Tensor, align: int = 16) -> torch.Tensor:
    """Contiguous copy whose data pointer meets the kernels' vector-load alignment."""
    t = t.contiguous()
    if t.data_ptr() % align:
        t = t.clone()
    return t
