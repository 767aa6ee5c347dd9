"""MLX-format safetensors loading of routed experts straight into HBM.

Mirrors ``SafetensorsMap`` of ``mlx_flash_compress/expert_streaming.py:60-168``
(header indexing, stacked ``[E, ...]`` tensors sliced per expert, the
per-expert ``experts.E.`` layout and Mixtral's ``w1/w2/w3`` naming) and the
weight keys of ``:576-583`` (``model.layers.L.mlp.switch_mlp.{gate,up,down}_proj
.{weight,scales,biases}``, ``block_sparse_moe`` for Mixtral).  Instead of
building host arrays per expert for a streaming cache, a rank loads the whole
``ExpertShard`` block of every layer once: the block's rows are one
contiguous byte range of a stacked tensor, read from the memory-mapped file
through a pinned staging buffer and copied to the device.

One deliberate difference: the reference maps safetensors ``BF16`` to NumPy
float16 (a reinterpretation of the bytes); here bf16 stays bf16.
"""

import json
import mmap
import os
import struct

import numpy as np
import torch

from .distributed_experts import ExpertShard

_DTYPES = {
    "BF16": (torch.bfloat16, 2),
    "F16": (torch.float16, 2),
    "F32": (torch.float32, 4),
    "U32": (torch.uint32, 4),
    "I32": (torch.int32, 4),
    "U8": (torch.uint8, 1),
}

_MIXTRAL_MAP = {"gate_proj": "w1", "down_proj": "w2", "up_proj": "w3"}
_STAGING_BYTES = 64 << 20


class SafetensorsMap:
    """Memory-mapped index of one or more safetensors shards."""

    def __init__(self, shard_paths):
        self._mmaps = {}
        self._files = {}
        self._tensors = {}  # key -> (path, dtype, shape, begin, end) with absolute file offsets
        for path in shard_paths:
            self._index_shard(path)

    def _index_shard(self, path):
        with open(path, "rb") as f:
            header_size = struct.unpack("<Q", f.read(8))[0]
            header = json.loads(f.read(header_size))
        start = 8 + header_size
        for key, info in header.items():
            if key == "__metadata__":
                continue
            b, e = info.get("data_offsets", [0, 0])
            self._tensors[key] = (path, info.get("dtype", "F16"), list(info.get("shape", [])), start + b, start + e)

    def _mm(self, path):
        if path not in self._mmaps:
            f = open(path, "rb")
            self._files[path] = f
            self._mmaps[path] = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        return self._mmaps[path]

    def has_key(self, key):
        return key in self._tensors

    def keys(self):
        return list(self._tensors)

    def _read(self, path, begin, end, dtype, shape, device):
        """Bytes [begin, end) of a shard as a tensor on `device` (pinned staging for CUDA)."""
        torch_dtype, _ = _DTYPES[dtype]
        mm = self._mm(path)
        raw = np.frombuffer(mm, dtype=np.uint8, count=end - begin, offset=begin)
        if device is None or torch.device(device).type == "cpu":
            return torch.from_numpy(raw.copy()).view(torch_dtype).reshape(shape)
        dev = torch.device(device)
        out = torch.empty(end - begin, dtype=torch.uint8, device=dev)
        stage = torch.empty(min(end - begin, _STAGING_BYTES), dtype=torch.uint8).pin_memory()
        stream = torch.cuda.current_stream(dev)
        for o in range(0, end - begin, stage.numel()):
            n = min(stage.numel(), end - begin - o)
            stream.synchronize()  # the staging buffer is free again
            stage[:n].numpy()[:] = raw[o:o + n]
            out[o:o + n].copy_(stage[:n], non_blocking=True)
        stream.synchronize()
        return out.view(torch_dtype).reshape(shape)

    def get_tensor(self, key, device=None):
        path, dtype, shape, b, e = self._tensors[key]
        return self._read(path, b, e, dtype, shape, device)

    def get_expert_slice(self, key, expert_ids, device=None):
        """Experts `expert_ids` of a stacked `[E, ...]` key, or of the per-expert /
        Mixtral layouts derived from it; None if the key is absent."""
        expert_ids = [int(e) for e in expert_ids]
        if key in self._tensors:
            path, dtype, shape, b, e = self._tensors[key]
            if len(shape) >= 3:
                row = (e - b) // shape[0]
                runs = _runs(expert_ids)
                parts = [self._read(path, b + lo * row, b + (hi + 1) * row, dtype, [hi + 1 - lo] + shape[1:], device)
                         for lo, hi in runs]
                return parts[0] if len(parts) == 1 else torch.cat(parts)
        per_expert = key.replace(".switch_mlp.", ".experts.0.")
        if per_expert not in self._tensors:
            for mlx_name, st_name in _MIXTRAL_MAP.items():
                per_expert = per_expert.replace(f".{mlx_name}.", f".{st_name}.")
        if per_expert in self._tensors:
            slices = []
            for eid in expert_ids:
                k = per_expert.replace(".experts.0.", f".experts.{eid}.")
                if k in self._tensors:
                    slices.append(self.get_tensor(k, device))
            if slices:
                return torch.stack(slices)
        return None

    def present_experts(self, key, expert_ids):
        """The ids among ``expert_ids`` whose tensors exist for ``key`` (every
        id for a stacked key, the ids with their own key in the per-expert and
        Mixtral layouts)."""
        expert_ids = [int(e) for e in expert_ids]
        if key in self._tensors:
            shape = self._tensors[key][2]
            return [e for e in expert_ids if len(shape) >= 3 and 0 <= e < shape[0]]
        per_expert = key.replace(".switch_mlp.", ".experts.0.")
        if per_expert not in self._tensors:
            for mlx_name, st_name in _MIXTRAL_MAP.items():
                per_expert = per_expert.replace(f".{mlx_name}.", f".{st_name}.")
        return [e for e in expert_ids if per_expert.replace(".experts.0.", f".experts.{e}.") in self._tensors]

    def close(self):
        for m in self._mmaps.values():
            m.close()
        for f in self._files.values():
            f.close()
        self._mmaps.clear()
        self._files.clear()


def _runs(ids):
    """Sorted ids grouped into contiguous [lo, hi] runs (order preserved when already sorted)."""
    runs = []
    for e in ids:
        if runs and e == runs[-1][1] + 1:
            runs[-1][1] = e
        else:
            runs.append([e, e])
    return [tuple(r) for r in runs]


def expert_weight_key(layer_idx, proj, suffix, mixtral=False):
    block = "block_sparse_moe" if mixtral else "mlp"
    return f"model.layers.{layer_idx}.{block}.switch_mlp.{proj}.{suffix}"


def load_moe_layer_shard(smap: SafetensorsMap, layer_idx: int, shard: ExpertShard, device, mixtral=False):
    """{proj: (wq, scales, biases)} of this rank's experts for one layer, on `device`."""
    owned = shard.owned_experts
    out = {}
    for proj in ("gate_proj", "up_proj", "down_proj"):
        parts = []
        for suffix in ("weight", "scales", "biases"):
            key = expert_weight_key(layer_idx, proj, suffix, mixtral)
            t = smap.get_expert_slice(key, owned, device)
            if t is None:
                raise KeyError(f"layer {layer_idx} {proj}.{suffix} not found")
            if t.shape[0] != len(owned):
                # a per-expert layout with some experts' keys absent: every later
                # expert's local index would shift, so refuse the shard
                have = set(smap.present_experts(key, owned))
                missing = [e for e in owned if e not in have]
                raise KeyError(f"layer {layer_idx} {proj}.{suffix}: experts {missing} not found")
            parts.append(t)
        out[proj] = tuple(parts)
    return out


def find_shards(model_dir):
    """The model's safetensors shards (sorted), as MLX-LM checkpoints name them."""
    files = sorted(f for f in os.listdir(model_dir) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {model_dir}")
    return [os.path.join(model_dir, f) for f in files]
