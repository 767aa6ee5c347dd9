"""MLX-format safetensors expert loading (host side, CPU): stacked [E, ...]
tensors sliced to an ExpertShard block, the per-expert `experts.E.` layout and
Mixtral's w1/w2/w3 naming (expert_streaming.py:60-168, :576-583)."""

import json
import struct

import numpy as np
import pytest
import torch

from b200flash.distributed_experts import ExpertShard
from b200flash.expert_loader import SafetensorsMap, expert_weight_key, load_moe_layer_shard

_ST = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}


def _write(path, tensors):
    header, blobs, off = {}, [], 0
    for k, a in tensors.items():
        a = np.ascontiguousarray(a)
        header[k] = {"dtype": _ST[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _layer(rng, E, N, K):
    return {"weight": rng.integers(0, 2**32, (E, N, K // 8), dtype=np.uint32),
            "scales": rng.integers(0, 2**16, (E, N, K // 64), dtype=np.uint16),
            "biases": rng.integers(0, 2**16, (E, N, K // 64), dtype=np.uint16)}


def test_stacked_layout_shard_slices(tmp_path):
    rng = np.random.default_rng(0)
    E, N, K = 10, 32, 128
    data = {p: _layer(rng, E, N, K) for p in ("gate_proj", "up_proj", "down_proj")}
    tensors = {expert_weight_key(0, p, s): data[p][s] for p in data for s in data[p]}
    path = str(tmp_path / "model.safetensors")
    _write(path, tensors)
    smap = SafetensorsMap([path])
    for W in (1, 3, 4):
        for r in range(W):
            shard = ExpertShard(rank=r, world_size=W, total_experts=E)
            got = load_moe_layer_shard(smap, 0, shard, None)
            lo, hi = shard.owned_experts[0], shard.owned_experts[-1] + 1
            for p in data:
                w, s, b = got[p]
                assert w.dtype == torch.uint32 and s.dtype == torch.bfloat16
                assert np.array_equal(w.view(torch.int32).numpy().view(np.uint32), data[p]["weight"][lo:hi])
                assert np.array_equal(s.view(torch.int16).numpy().view(np.uint16), data[p]["scales"][lo:hi])
    # non-contiguous ids come back in the requested order
    got = smap.get_expert_slice(expert_weight_key(0, "up_proj", "weight"), [7, 2, 3], None)
    assert np.array_equal(got.view(torch.int32).numpy().view(np.uint32), data["up_proj"]["weight"][[7, 2, 3]])
    smap.close()


@pytest.mark.parametrize("mixtral", [False, True])
def test_per_expert_layouts(tmp_path, mixtral):
    rng = np.random.default_rng(1)
    E, N, K = 4, 16, 128
    data = {p: _layer(rng, E, N, K) for p in ("gate_proj", "up_proj", "down_proj")}
    names = {"gate_proj": "w1", "down_proj": "w2", "up_proj": "w3"}
    block = "block_sparse_moe" if mixtral else "mlp"
    tensors = {}
    for p in data:
        for s in data[p]:
            for e in range(E):
                pn = names[p] if mixtral else p
                tensors[f"model.layers.2.{block}.experts.{e}.{pn}.{s}"] = data[p][s][e]
    path = str(tmp_path / "per_expert.safetensors")
    _write(path, tensors)
    smap = SafetensorsMap([path])
    shard = ExpertShard(rank=1, world_size=2, total_experts=E)
    got = load_moe_layer_shard(smap, 2, shard, None, mixtral=mixtral)
    for p in data:
        assert np.array_equal(got[p][0].view(torch.int32).numpy().view(np.uint32), data[p]["weight"][2:4])
    with pytest.raises(KeyError):
        load_moe_layer_shard(smap, 3, shard, None, mixtral=mixtral)
    smap.close()


def test_per_expert_layout_missing_expert_is_refused(tmp_path):
    """An expert whose per-expert keys are absent must not shift the local
    indices of the experts after it: the shard load names the missing ids."""
    rng = np.random.default_rng(2)
    E, N, K = 4, 16, 128
    data = {p: _layer(rng, E, N, K) for p in ("gate_proj", "up_proj", "down_proj")}
    tensors = {f"model.layers.0.mlp.experts.{e}.{p}.{s}": data[p][s][e]
               for p in data for s in data[p] for e in range(E) if e != 2}
    path = str(tmp_path / "gap.safetensors")
    _write(path, tensors)
    smap = SafetensorsMap([path])
    with pytest.raises(KeyError, match=r"experts \[2\]"):
        load_moe_layer_shard(smap, 0, ExpertShard(rank=0, world_size=1, total_experts=E), None)
    # a shard that does not own the gap still loads
    got = load_moe_layer_shard(smap, 0, ExpertShard(rank=0, world_size=2, total_experts=E), None)
    assert got["up_proj"][0].shape[0] == 2
    smap.close()


@pytest.mark.gpu
def test_loaded_shard_drives_the_expert_kernels(tmp_path, dev):
    """Quantized experts written as MLX safetensors, loaded to HBM for one
    shard, then used by the grouped GEMV: same outputs as the oracle."""
    from b200flash import mx_compat
    from oracle import affine
    from oracle.fp import bf16_bits, round_to

    from helpers import assert_close, to_dev, to_np

    rng = np.random.default_rng(3)
    E, N, K, T, k = 6, 64, 256, 5, 2
    w = round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16")
    wq, s, b = affine.quantize(w, 64, 4)
    tensors = {expert_weight_key(0, p, "weight"): wq for p in ("gate_proj", "up_proj", "down_proj")}
    for p in ("gate_proj", "up_proj", "down_proj"):
        tensors[expert_weight_key(0, p, "scales")] = bf16_bits(s)
        tensors[expert_weight_key(0, p, "biases")] = bf16_bits(b)
    path = str(tmp_path / "q.safetensors")
    _write(path, tensors)
    smap = SafetensorsMap([path])
    shard = ExpertShard(rank=1, world_size=2, total_experts=E)  # experts 3..5
    got = load_moe_layer_shard(smap, 0, shard, dev)
    gw, gs, gb = got["gate_proj"]
    assert gw.is_cuda and gs.dtype == torch.bfloat16
    x = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    inds = rng.integers(0, 3, (T, k)).astype(np.int32)  # local expert ids
    out = mx_compat.gather_qmm(to_dev(x, "bf16", dev), gw, gs, gb, rhs_indices=torch.from_numpy(inds).to(dev),
                               transpose=True, group_size=64, bits=4)
    want = affine.gather_qmm(x, wq[3:], s[3:], b[3:], rhs_indices=inds, group_size=64, bits=4, out_dtype="f32")
    assert_close(to_np(out), want, what="gather_qmm over loaded shard")
    smap.close()
