"""Quantized KV cache -- drop-in for ``mlx_flash_compress/quantized_kv_cache.py``.

Same public names, signatures, error messages and numbers as the reference
(``quantize_tensor`` / ``dequantize_tensor`` are byte-exact), running on CUDA
torch tensors through libb200flash:

* ``quantize_tensor``    -> ``b2f_kv_quantize_sym``   (quantized_kv_cache.py:68-156)
* ``dequantize_tensor``  -> ``b2f_kv_dequantize_sym`` (quantized_kv_cache.py:159-234)
* ``QuantizedKVEntry``   keeps the reference's calibration and chunk semantics
  (quantized_kv_cache.py:237-388) but stores the quantized chunks back to back
  in one growable token-major buffer, so ``get_keys_values`` is a single
  dequantize launch instead of a Python loop over chunks, and ``attend`` runs
  the fused quantized-KV decode attention without materialising fp32 K/V.
"""

from dataclasses import dataclass
from typing import Optional

import torch

from . import _capi
from ._capi import DTYPE_CODES, call, ptr, require_cuda, stream_of


@dataclass
class QuantizedKVConfig:
    """Configuration for quantized KV cache (quantized_kv_cache.py:39-65)."""

    key_bits: int = 4
    value_bits: int = 4
    group_size: int = 64
    calibration_tokens: int = 32

    def __post_init__(self):
        if self.key_bits not in (2, 4, 8):
            raise ValueError(f"key_bits must be 2, 4, or 8, got {self.key_bits}")
        if self.value_bits not in (2, 4, 8):
            raise ValueError(f"value_bits must be 2, 4, or 8, got {self.value_bits}")
        if self.group_size <= 0:
            raise ValueError(f"group_size must be positive, got {self.group_size}")
        if self.calibration_tokens < 0:
            raise ValueError(f"calibration_tokens must be non-negative, got {self.calibration_tokens}")


def packed_len(D: int, bits: int, group_size: int) -> int:
    return int(_capi.lib().b2f_kv_packed_len(D, bits, group_size))


def num_groups(D: int, group_size: int) -> int:
    return int(_capi.lib().b2f_kv_num_groups(D, group_size))


def _quantize_rows_into(x2d, bits, group_size, packed, packed_ld, scales, scales_ld, dst_row=None, zeros=None):
    dev = require_cuda(x2d, packed, scales)
    rows, D = x2d.shape
    call("b2f_kv_quantize_sym", ptr(x2d), DTYPE_CODES[x2d.dtype], rows, D, bits, group_size, ptr(dst_row),
         ptr(packed), packed_ld, ptr(scales), ptr(zeros), scales_ld, stream_of(dev))


def quantize_tensor(x: torch.Tensor, bits: int, group_size: int = 64):
    """Per-group absmax quantization -> ``(packed uint8, scales f32, zeros f32)``."""
    if bits not in (2, 4, 8):
        raise ValueError(f"bits must be 2, 4, or 8, got {bits}")
    if group_size <= 0:
        raise ValueError(f"group_size must be positive, got {group_size}")
    shape = tuple(x.shape)
    if not shape or shape[-1] == 0:
        e = torch.zeros((0,), dtype=torch.float32, device=x.device)
        return torch.zeros((0,), dtype=torch.uint8, device=x.device), e, e.clone()
    if x.dtype not in DTYPE_CODES:
        raise ValueError(f"unsupported dtype {x.dtype}")
    dev = require_cuda(x)
    D = shape[-1]
    lead = shape[:-1]
    pl = packed_len(D, bits, group_size)
    ng = num_groups(D, group_size)
    x2 = x.reshape(-1, D).contiguous()
    packed = torch.empty(*lead, pl, dtype=torch.uint8, device=dev)
    scales = torch.empty(*lead, ng, dtype=torch.float32, device=dev)
    zeros = torch.empty_like(scales)
    _quantize_rows_into(x2, bits, group_size, packed, pl, scales, ng, zeros=zeros)
    return packed, scales, zeros


def dequantize_tensor(quantized: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, bits: int,
                      original_shape: tuple, group_size: int = 64) -> torch.Tensor:
    """Inverse of :func:`quantize_tensor`; returns float32 of ``original_shape``."""
    if bits not in (2, 4, 8):
        raise ValueError(f"bits must be 2, 4, or 8, got {bits}")
    original_shape = tuple(original_shape)
    if not original_shape or original_shape[-1] == 0:
        return torch.zeros(original_shape, dtype=torch.float32, device=quantized.device)
    dev = require_cuda(quantized, scales)
    D = original_shape[-1]
    rows = 1
    for d in original_shape[:-1]:
        rows *= d
    q = quantized.reshape(rows, -1).contiguous()
    s = scales.reshape(rows, -1).contiguous()
    out = torch.empty(original_shape, dtype=torch.float32, device=dev)
    call("b2f_kv_dequantize_sym", ptr(q), q.shape[1], ptr(s), s.shape[1], 0, rows, D, bits, group_size,
         ptr(out), stream_of(dev))
    return out


def decode_attention(q: torch.Tensor, k_pages: torch.Tensor, k_scales: torch.Tensor, v_pages: torch.Tensor,
                     v_scales: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor, bits: int,
                     page_size: int, num_kv_heads: int, softmax_scale: Optional[float] = None,
                     group_size: int = 64, token_major: bool = False,
                     n_splits: Optional[int] = None) -> torch.Tensor:
    """Fused decode attention over packed K/V pages (kernel ``b2f_qkv_decode_attn``).

    ``q``: bf16 ``[B, Hq, D]``.  ``k_pages``/``v_pages``: uint8 with
    ``Hkv*page_size`` rows of ``packed_len(D)`` bytes per page; scales f32 with
    ``D/64`` per row.  Pages are head-major (``[page][Hkv][slot]``) unless
    ``token_major`` (``[page][slot][Hkv]``, the reference's chunk order).
    """
    dev = require_cuda(q, k_pages, k_scales, v_pages, v_scales, block_table, seq_lens)
    if q.dtype != torch.bfloat16:
        raise ValueError("q must be bf16")
    B, Hq, D = q.shape
    Hkv = int(num_kv_heads)
    if Hkv <= 0 or Hq % Hkv:
        raise ValueError(f"num_kv_heads {Hkv} must divide the {Hq} query heads")
    if k_pages.numel() < int(block_table.max().item() + 1) * Hkv * page_size * packed_len(D, bits, group_size):
        raise ValueError("block_table points past the end of the page pool")
    if softmax_scale is None:
        softmax_scale = D ** -0.5
    if n_splits is None:
        n_splits = pick_splits(B, Hkv, int(seq_lens.max().item()) if seq_lens.numel() else 0)
    bt = block_table.to(torch.int32).contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
    ws_bytes = int(_capi.lib().b2f_qkv_decode_attn_workspace_bytes(B, Hq, D, n_splits))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev) if ws_bytes else None
    hs, ss = (1, Hkv) if token_major else (page_size, 1)
    call("b2f_qkv_decode_attn", ptr(q.contiguous()), ptr(k_pages), ptr(k_scales), ptr(v_pages), ptr(v_scales),
         ptr(bt), bt.shape[1], ptr(sl), B, Hq, Hkv, D, page_size, hs, ss, bits, group_size,
         float(softmax_scale), n_splits, ptr(ws), ws_bytes, ptr(out), stream_of(dev))
    return out


def pick_splits(B: int, Hkv: int, max_len: int, sms: int = 148) -> int:
    """Context splits: about two CTAs per SM, at least 256 tokens per split.
    Measured on B200 (8-bit KV, 32q/4kv heads of 128, context 2048): batch 1
    24.4 us unsplit -> 10.3 us with 8 splits; batch 8 24.9 -> 12.3 us; batch
    64 fastest unsplit (34.9 us; 2 splits 43.5)."""
    if max_len <= 0:
        return 1
    want = max(1, (2 * sms) // max(1, B * Hkv))
    cap = max(1, max_len // 256)
    return int(min(want, cap, 64))


class QuantizedKVEntry:
    """One layer's quantized KV cache (quantized_kv_cache.py:237-388).

    Tokens ``[0, calibration_tokens)`` stay in full precision until the
    calibration window closes; then everything is quantized, and later
    appends are quantized immediately.  Quantized rows live in a token-major
    buffer ``[capacity, H, packed_len]`` (+ f32 scales), one row per
    (token, head) exactly as ``quantize_tensor`` lays them out.
    """

    PAGE = 16

    def __init__(self, num_heads: int, head_dim: int, config: QuantizedKVConfig):
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.config = config
        self._fp_keys: Optional[torch.Tensor] = None
        self._fp_values: Optional[torch.Tensor] = None
        self._chunks: list = []  # (t0, t1, shape)
        self._length = 0
        self._qlen = 0
        self._calibration_done = False
        self._cap = 0
        self._kp = self._ks = self._vp = self._vs = None
        self._kpl = packed_len(head_dim, config.key_bits, config.group_size)
        self._vpl = packed_len(head_dim, config.value_bits, config.group_size)
        self._ng = num_groups(head_dim, config.group_size)

    # -- storage --------------------------------------------------------------
    def _ensure(self, tokens: int, device):
        if tokens <= self._cap:
            return
        cap = max(self.PAGE, self._cap)
        while cap < tokens:
            cap *= 2
        H = self.num_heads
        kp = torch.empty(cap, H, self._kpl, dtype=torch.uint8, device=device)
        vp = torch.empty(cap, H, self._vpl, dtype=torch.uint8, device=device)
        ks = torch.empty(cap, H, self._ng, dtype=torch.float32, device=device)
        vs = torch.empty(cap, H, self._ng, dtype=torch.float32, device=device)
        if self._qlen:
            kp[: self._qlen].copy_(self._kp[: self._qlen])
            vp[: self._qlen].copy_(self._vp[: self._qlen])
            ks[: self._qlen].copy_(self._ks[: self._qlen])
            vs[: self._qlen].copy_(self._vs[: self._qlen])
        self._kp, self._vp, self._ks, self._vs, self._cap = kp, vp, ks, vs, cap

    def _store(self, keys: torch.Tensor, values: torch.Tensor):
        S = keys.shape[0]
        t0 = self._qlen
        self._ensure(t0 + S, keys.device)
        H, D = self.num_heads, self.head_dim
        gs = self.config.group_size
        _quantize_rows_into(keys.reshape(S * H, D).contiguous(), self.config.key_bits, gs,
                            self._kp[t0:], self._kpl, self._ks[t0:], self._ng)
        _quantize_rows_into(values.reshape(S * H, D).contiguous(), self.config.value_bits, gs,
                            self._vp[t0:], self._vpl, self._vs[t0:], self._ng)
        self._qlen = t0 + S
        self._chunks.append((t0, t0 + S, tuple(keys.shape)))

    def _chunk_views(self, packed, scales):
        out = []
        for t0, t1, shape in self._chunks:
            s = scales[t0:t1]
            out.append((packed[t0:t1], s, torch.zeros((), device=s.device).expand_as(s), shape))
        return out

    @property
    def _q_keys(self):
        return self._chunk_views(self._kp, self._ks) if self._chunks else []

    @property
    def _q_values(self):
        return self._chunk_views(self._vp, self._vs) if self._chunks else []

    # -- reference API ----------------------------------------------------------
    def _finalize_calibration(self):
        if self._fp_keys is None:
            self._calibration_done = True
            return
        self._store(self._fp_keys, self._fp_values)
        self._fp_keys = None
        self._fp_values = None
        self._calibration_done = True

    def append(self, keys: torch.Tensor, values: torch.Tensor):
        """Append ``keys``/``values`` of shape ``(seq_len, num_heads, head_dim)``."""
        seq_len = keys.shape[0]
        self._length += seq_len
        if not self._calibration_done:
            if self._fp_keys is None:
                self._fp_keys = keys
                self._fp_values = values
            else:
                self._fp_keys = torch.cat([self._fp_keys, keys], dim=0)
                self._fp_values = torch.cat([self._fp_values, values], dim=0)
            if self._length >= self.config.calibration_tokens:
                self._finalize_calibration()
        else:
            self._store(keys, values)

    def get_keys_values(self):
        """Full K/V as float32 ``(total_seq, num_heads, head_dim)``."""
        if not self._calibration_done:
            if self._fp_keys is None:
                raise ValueError("No data in cache")
            return self._fp_keys.to(torch.float32), self._fp_values.to(torch.float32)
        if not self._chunks:
            raise ValueError("No data in cache")
        n, H, D = self._qlen, self.num_heads, self.head_dim
        gs = self.config.group_size
        dev = self._kp.device
        k = torch.empty(n, H, D, dtype=torch.float32, device=dev)
        v = torch.empty(n, H, D, dtype=torch.float32, device=dev)
        call("b2f_kv_dequantize_sym", ptr(self._kp), self._kpl, ptr(self._ks), self._ng, 0, n * H, D,
             self.config.key_bits, gs, ptr(k), stream_of(dev))
        call("b2f_kv_dequantize_sym", ptr(self._vp), self._vpl, ptr(self._vs), self._ng, 0, n * H, D,
             self.config.value_bits, gs, ptr(v), stream_of(dev))
        return k, v

    def attend(self, q: torch.Tensor, softmax_scale: Optional[float] = None) -> torch.Tensor:
        """Fused decode attention of ``q`` (bf16 ``[Hq, D]``) over the quantized cache."""
        if not self._calibration_done or not self._chunks:
            raise ValueError("fused attention needs a quantized cache (calibration finished)")
        if self.config.key_bits != self.config.value_bits:
            raise ValueError("fused attention needs key_bits == value_bits")
        dev = self._kp.device
        npages = self._cap // self.PAGE
        bt = torch.arange(npages, dtype=torch.int32, device=dev).reshape(1, npages)
        sl = torch.tensor([self._qlen], dtype=torch.int32, device=dev)
        out = decode_attention(q.reshape(1, *q.shape[-2:]), self._kp, self._ks, self._vp, self._vs, bt, sl,
                               self.config.key_bits, self.PAGE, self.num_heads, softmax_scale,
                               self.config.group_size, token_major=True)
        return out.reshape(q.shape)

    @property
    def length(self) -> int:
        return self._length

    @property
    def memory_bytes(self) -> int:
        """Memory as the reference accounts it (fp16 calibration data; packed
        bytes + float32 scales + float32 zeros per quantized chunk)."""
        total = 0
        if self._fp_keys is not None:
            total += self._fp_keys.numel() * 2 + self._fp_values.numel() * 2
        rows = self._qlen * self.num_heads
        total += rows * (self._kpl + self._vpl) + 2 * rows * self._ng * 8
        return total

    @property
    def full_precision_bytes(self) -> int:
        return self._length * self.num_heads * self.head_dim * 2 * 2


class QuantizedKVCacheManager:
    """Per-layer quantized KV caches (quantized_kv_cache.py:391-497)."""

    def __init__(self, config: QuantizedKVConfig, num_layers: int, num_kv_heads: int, head_dim: int):
        if num_layers <= 0:
            raise ValueError(f"num_layers must be positive, got {num_layers}")
        if num_kv_heads <= 0:
            raise ValueError(f"num_kv_heads must be positive, got {num_kv_heads}")
        if head_dim <= 0:
            raise ValueError(f"head_dim must be positive, got {head_dim}")
        self.config = config
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.entries = [QuantizedKVEntry(num_kv_heads, head_dim, config) for _ in range(num_layers)]

    def _check(self, layer_idx):
        if layer_idx < 0 or layer_idx >= self.num_layers:
            raise IndexError(f"layer_idx {layer_idx} out of range [0, {self.num_layers})")

    def update(self, layer_idx: int, keys: torch.Tensor, values: torch.Tensor):
        self._check(layer_idx)
        self.entries[layer_idx].append(keys, values)

    def get_kv(self, layer_idx: int):
        self._check(layer_idx)
        return self.entries[layer_idx].get_keys_values()

    def attend(self, layer_idx: int, q: torch.Tensor, softmax_scale: Optional[float] = None):
        """Fused quantized-KV decode attention for one query token ``[Hq, D]``."""
        self._check(layer_idx)
        return self.entries[layer_idx].attend(q, softmax_scale)

    def get_compression_ratio(self) -> float:
        total_actual = sum(e.memory_bytes for e in self.entries)
        total_fp = sum(e.full_precision_bytes for e in self.entries)
        if total_fp == 0:
            return 1.0
        return total_actual / total_fp

    def get_stats(self) -> dict:
        total_actual = sum(e.memory_bytes for e in self.entries)
        total_fp = sum(e.full_precision_bytes for e in self.entries)
        total_tokens = sum(e.length for e in self.entries)
        per_layer = []
        for i, entry in enumerate(self.entries):
            fp = entry.full_precision_bytes
            actual = entry.memory_bytes
            per_layer.append({
                "layer": i,
                "tokens": entry.length,
                "memory_bytes": actual,
                "full_precision_bytes": fp,
                "compression_ratio": actual / fp if fp > 0 else 1.0,
                "calibration_done": entry._calibration_done,
            })
        return {
            "config": {
                "key_bits": self.config.key_bits,
                "value_bits": self.config.value_bits,
                "group_size": self.config.group_size,
                "calibration_tokens": self.config.calibration_tokens,
            },
            "num_layers": self.num_layers,
            "total_tokens": total_tokens,
            "total_memory_bytes": total_actual,
            "total_full_precision_bytes": total_fp,
            "compression_ratio": total_actual / total_fp if total_fp > 0 else 1.0,
            "memory_savings_pct": round((1.0 - total_actual / total_fp) * 100, 1) if total_fp > 0 else 0.0,
            "per_layer": per_layer,
        }

    def reset(self):
        self.entries = [QuantizedKVEntry(self.num_kv_heads, self.head_dim, self.config)
                        for _ in range(self.num_layers)]


def apply_quantized_kv_cache(model, config: Optional[QuantizedKVConfig] = None) -> QuantizedKVCacheManager:
    """Detect layers / kv heads / head_dim on ``model`` and build a manager
    (quantized_kv_cache.py:500-566)."""
    if config is None:
        config = QuantizedKVConfig()
    num_layers = num_kv_heads = head_dim = 0
    if hasattr(model, "layers"):
        layers = model.layers
        num_layers = len(layers)
        if num_layers > 0:
            layer0 = layers[0]
            attn = None
            for name in ("self_attn", "attention", "attn"):
                if hasattr(layer0, name):
                    attn = getattr(layer0, name)
                    break
            if attn is not None:
                for name in ("n_kv_heads", "num_kv_heads", "n_heads_kv"):
                    if hasattr(attn, name):
                        num_kv_heads = getattr(attn, name)
                        break
                if num_kv_heads == 0:
                    for name in ("n_heads", "num_heads"):
                        if hasattr(attn, name):
                            num_kv_heads = getattr(attn, name)
                            break
                for name in ("head_dim", "d_head"):
                    if hasattr(attn, name):
                        head_dim = getattr(attn, name)
                        break
    elif hasattr(model, "n_layers"):
        num_layers = model.n_layers
    if num_layers == 0:
        raise ValueError("Could not detect model architecture. Model must have a 'layers' attribute.")
    if num_kv_heads == 0 or head_dim == 0:
        raise ValueError(
            "Could not detect num_kv_heads or head_dim from model. "
            "Provide these values manually via QuantizedKVCacheManager.")
    return QuantizedKVCacheManager(config=config, num_layers=num_layers, num_kv_heads=num_kv_heads,
                                   head_dim=head_dim)
