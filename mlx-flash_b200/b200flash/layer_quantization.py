"""Drop-in for ``mlx_flash_compress/layer_quantization.py`` on torch modules.

* ``QuantizedLinear.from_linear`` (the ``nn.QuantizedLinear.from_linear``
  call at ``layer_quantization.py:254``): packs the weight with
  ``b2f_quantize_affine`` and runs the forward through ``b2f_qgemv_affine``
  (decode-sized inputs) or the tcgen05 GEMM (prefill-sized, group 64).
* ``LayerSensitivityProfile`` (``:52-185``): per-layer output MSE under a
  per-tensor symmetric fake quantization of the layer's linears, done by
  ``b2f_fake_quant_sym`` (``_quantize_linears_inplace``, ``:461-494``).
* ``LayerQuantizer``, ``apply_layer_quantization``, ``estimate_model_size``
  (``:188-379``): precision maps (first/last layers at 8 bits by default) and
  the in-place replacement of every linear by a ``QuantizedLinear``.

Layers are found as ``model.model.layers`` or ``model.layers``; linears at
the standard ``self_attn.{q,k,v,o}_proj`` / ``mlp.{gate,up,down}_proj``
paths, else by a recursive search (``:382-437``).
"""

import time
from dataclasses import dataclass, field
from typing import Any

import torch

from . import mx_compat
from ._capi import call, ptr, require_cuda, stream_of

_DT = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


@dataclass
class LayerQuantConfig:
    default_bits: int = 4
    sensitive_bits: int = 8
    sensitive_layers: list = field(default_factory=list)
    num_sensitive_start: int = 2
    num_sensitive_end: int = 2
    group_size: int = 64
    calibration_samples: int = 32


def _get_layers(model):
    if hasattr(model, "model") and hasattr(model.model, "layers"):
        return model.model.layers
    if hasattr(model, "layers"):
        return model.layers
    raise AttributeError("Cannot find model layers (tried model.model.layers and model.layers)")


class QuantizedLinear(torch.nn.Module):
    """Affine group-quantized linear: ``y = x @ dequantize(wq).T (+ bias)``."""

    def __init__(self, wq, scales, biases, bias=None, group_size: int = 64, bits: int = 4):
        super().__init__()
        self.register_buffer("weight", wq)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.bias = None if bias is None else torch.nn.Parameter(bias.detach().to(torch.bfloat16),
                                                                 requires_grad=False)
        self.group_size, self.bits = group_size, bits
        self.out_features = wq.shape[0]
        self.in_features = wq.shape[1] * 32 // bits

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, group_size: int = 64, bits: int = 4) -> "QuantizedLinear":
        w = linear.weight.detach()
        require_cuda(w)
        wq, s, b = mx_compat.quantize(w.to(torch.bfloat16), group_size=group_size, bits=bits)
        return cls(wq, s, b, linear.bias, group_size, bits)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xb = x.to(torch.bfloat16)
        M = xb.numel() // self.in_features
        if M >= 64 and self.bits in (4, 8) and mx_compat.tc_supported(self.in_features, self.group_size, self.bits):
            y = mx_compat.quantized_matmul_tc(xb.reshape(M, self.in_features), self.weight, self.scales,
                                              self.biases, self.group_size, self.bits)
            y = y.reshape(*xb.shape[:-1], self.out_features)
        else:
            y = mx_compat.quantized_matmul(xb, self.weight, self.scales, self.biases, True, self.group_size,
                                           self.bits)
        if self.bias is not None:
            y = y + self.bias
        return y


def fake_quantize_sym(w: torch.Tensor, bits: int = 4):
    """Per-tensor symmetric absmax quantize-dequantize (layer_quantization.py:461-494).

    Returns ``(fp32 tensor of w's shape, fp32 absmax)``: ``scale =
    max(absmax/qmax in w's dtype, 1e-10)``, ``out = clip(rint(w/scale), qmin,
    qmax) * scale`` with ``(qmin, qmax) = (-8, 7)`` at 4 bits, ``(-128, 127)``
    at 8 bits.
    """
    dev = require_cuda(w)
    if w.dtype not in _DT:
        raise ValueError(f"unsupported dtype {w.dtype}")
    wc = w.detach().contiguous()
    out = torch.empty(wc.shape, dtype=torch.float32, device=dev)
    amax = torch.empty(1, dtype=torch.float32, device=dev)
    call("b2f_fake_quant_sym", ptr(wc), _DT[wc.dtype], wc.numel(), 4 if bits <= 4 else 8, ptr(out), ptr(amax),
         stream_of(dev))
    return out, amax


def _get_nested_attr(module, dotted: str):
    cur = module
    for part in dotted.split("."):
        if not hasattr(cur, part):
            return None
        cur = getattr(cur, part)
    return cur


def _set_nested_attr(module, dotted: str, value):
    parts = dotted.split(".")
    cur = module
    for part in parts[:-1]:
        cur = getattr(cur, part)
    setattr(cur, parts[-1], value)


_STANDARD = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
             "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def _find_linear_layers(module: torch.nn.Module) -> list:
    found = []
    for path in _STANDARD:
        sub = _get_nested_attr(module, path)
        if isinstance(sub, torch.nn.Linear):
            found.append((path, sub))
    if not found:
        found = [(n, m) for n, m in module.named_modules() if n and isinstance(m, torch.nn.Linear)]
    return found


def _quantize_linears_inplace(linears: list, bits: int, group_size: int):
    """Bake the fake-quantization error into each linear's weight (fp32, as MLX promotes it)."""
    for _name, lin in linears:
        fq, _ = fake_quantize_sym(lin.weight, bits)
        lin.weight = torch.nn.Parameter(fq, requires_grad=False)


def _count_linear_params(module) -> int:
    return sum(lin.weight.shape[0] * lin.weight.shape[1] for _, lin in _find_linear_layers(module))


class LayerSensitivityProfile:
    def __init__(self, num_layers: int):
        self.num_layers = num_layers
        self.sensitivity_scores: list = []

    def measure_sensitivity(self, model, calibration_data: torch.Tensor) -> list:
        layers = _get_layers(model)
        self.sensitivity_scores = [self._measure_layer_sensitivity(layers[i], calibration_data)
                                   for i in range(self.num_layers)]
        return self.sensitivity_scores

    @torch.no_grad()
    def _measure_layer_sensitivity(self, layer, calibration_data) -> float:
        linears = _find_linear_layers(layer)
        if not linears:
            return 0.0
        original = layer(calibration_data)
        saved = {name: lin.weight for name, lin in linears}
        _quantize_linears_inplace(linears, bits=4, group_size=64)
        quantized = layer(calibration_data)
        diff = original.float() - quantized.float()
        mse = float((diff * diff).mean().item())
        for name, lin in linears:
            lin.weight = saved[name]
        return mse

    def get_precision_map(self, config: LayerQuantConfig = None) -> dict:
        config = config or LayerQuantConfig()
        if not self.sensitivity_scores:
            return self.default_precision_map(self.num_layers, config)
        if config.sensitive_layers:
            return {i: config.sensitive_bits if i in config.sensitive_layers else config.default_bits
                    for i in range(self.num_layers)}
        srt = sorted(self.sensitivity_scores)
        ti = int(len(srt) * 0.75)
        thr = srt[ti] if ti < len(srt) else 0.0
        return {i: config.sensitive_bits if (sc >= thr and thr > 0) else config.default_bits
                for i, sc in enumerate(self.sensitivity_scores)}

    @staticmethod
    def default_precision_map(num_layers: int, config: LayerQuantConfig = None) -> dict:
        config = config or LayerQuantConfig()
        pm = {}
        for i in range(num_layers):
            edge = i < config.num_sensitive_start or i >= num_layers - config.num_sensitive_end
            pm[i] = config.sensitive_bits if edge else config.default_bits
        return pm


class LayerQuantizer:
    def __init__(self, config: LayerQuantConfig = None):
        self.config = config or LayerQuantConfig()
        self._stats: dict[str, Any] = {"layers_quantized": 0, "layers_skipped": 0, "linears_quantized": 0,
                                       "bits_distribution": {}, "elapsed_ms": 0.0}

    def quantize_model(self, model, precision_map: dict = None) -> dict:
        layers = _get_layers(model)
        n = len(layers)
        if precision_map is None:
            precision_map = LayerSensitivityProfile.default_precision_map(n, self.config)
        t0 = time.monotonic()
        self._stats["bits_distribution"] = {}
        for i in range(n):
            bits = precision_map.get(i, self.config.default_bits)
            self._stats["bits_distribution"][i] = bits
            self.quantize_layer(layers[i], bits=bits, group_size=self.config.group_size)
            self._stats["layers_quantized"] += 1
        self._stats["elapsed_ms"] = (time.monotonic() - t0) * 1000
        return {"num_layers": n, "precision_map": precision_map, "stats": self.get_stats()}

    def quantize_layer(self, layer, bits: int, group_size: int = 64):
        for name, lin in _find_linear_layers(layer):
            _set_nested_attr(layer, name, QuantizedLinear.from_linear(lin, group_size=group_size, bits=bits))
            self._stats["linears_quantized"] += 1

    def estimate_memory_savings(self, model, precision_map: dict) -> dict:
        layers = _get_layers(model)
        total = 0
        uni = mixed = 0.0
        for i in range(len(layers)):
            p = _count_linear_params(layers[i])
            total += p
            uni += p * 4 / 8
            mixed += p * precision_map.get(i, self.config.default_bits) / 8
        sav = uni - mixed
        return {"total_params": total, "num_layers": len(layers), "uniform_q4_bytes": uni, "mixed_bytes": mixed,
                "savings_bytes": sav, "savings_ratio": sav / uni if uni > 0 else 0.0,
                "precision_map": precision_map, "effective_bits": mixed * 8 / total if total > 0 else 0.0}

    def get_stats(self) -> dict:
        return dict(self._stats)


def apply_layer_quantization(model, config: LayerQuantConfig = None, profile: bool = False,
                             calibration_data: torch.Tensor = None) -> dict:
    config = config or LayerQuantConfig()
    n = len(model.model.layers)
    if profile:
        if calibration_data is None:
            raise ValueError("calibration_data is required when profile=True")
        prof = LayerSensitivityProfile(n)
        scores = prof.measure_sensitivity(model, calibration_data)
        pm = prof.get_precision_map(config)
        pres = {"sensitivity_scores": scores, "profiled": True}
    else:
        pm = LayerSensitivityProfile.default_precision_map(n, config)
        pres = {"profiled": False}
    q = LayerQuantizer(config)
    # sizes are counted from the float linears, before they are replaced
    memory = q.estimate_memory_savings(model, pm)
    result = q.quantize_model(model, pm)
    result["profiling"] = pres
    result["memory"] = memory
    return result


def estimate_model_size(model, precision_map: dict) -> dict:
    return LayerQuantizer().estimate_memory_savings(model, precision_map)
