"""b200flash: B200 (sm_100a) kernels for MLX-Flash's quantized-weight and
quantized-KV-cache hot path, behind the reference's Python signatures.

Compute goes through libb200flash.so (C ABI in include/b2f.h); PyTorch only
owns device memory and streams.  There is no CPU fallback.
"""

__version__ = "0.1.0"

from ._capi import B2FError, lib  # noqa: F401
from .mx_compat import dequantize, gather_qmm, quantize, quantized_matmul  # noqa: F401
from .quantized_kv_cache import (  # noqa: F401
    QuantizedKVCacheManager,
    QuantizedKVConfig,
    QuantizedKVEntry,
    apply_quantized_kv_cache,
    decode_attention,
    dequantize_tensor,
    quantize_tensor,
)
