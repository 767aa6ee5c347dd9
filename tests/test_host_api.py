"""Host-side logic of the drop-in API (no GPU needed)."""

import json
import os

import pytest
import torch

from b200flash.distributed_experts import DistributedConfig, ExpertShard, plan_expert_distribution
from b200flash.quantized_kv_cache import QuantizedKVConfig, dequantize_tensor, quantize_tensor

from conftest import GOLDEN


def test_expert_shard_matches_reference_fixture():
    with open(os.path.join(GOLDEN, "ep_shard.json")) as f:
        rows = json.load(f)
    for row in rows:
        s = ExpertShard(rank=row["rank"], world_size=row["W"], total_experts=row["E"])
        assert s.owned_experts == row["owned"], row
        assert s.owner_table() == row["owners"], row


def test_expert_shard_reference_cases():
    assert ExpertShard(rank=2, world_size=3, total_experts=10).owned_experts == list(range(6, 10))
    s = ExpertShard(rank=0, world_size=2, total_experts=10)
    assert s.is_local(4) and not s.is_local(5)
    assert ExpertShard(rank=0, world_size=100, total_experts=2).owner_of(1) == 0
    st = ExpertShard(rank=0, world_size=1, total_experts=0, owned_experts=[]).stats()
    assert st["expert_range"] == "none"
    assert "0-29" in ExpertShard(rank=0, world_size=2, total_experts=60).stats()["expert_range"]


def test_distributed_config_env(monkeypatch):
    monkeypatch.setenv("MLX_WORLD_SIZE", "4")
    monkeypatch.setenv("MLX_RANK", "2")
    c = DistributedConfig.from_env()
    assert (c.world_size, c.rank, c.is_distributed, c.is_main) == (4, 2, True, False)
    p = plan_expert_distribution(128, 48, 8)
    assert p["experts_per_node"] == 16 and len(p["nodes"]) == 8


def test_kv_config_validation_messages():
    with pytest.raises(ValueError, match="key_bits must be 2, 4, or 8"):
        QuantizedKVConfig(key_bits=3)
    with pytest.raises(ValueError, match="value_bits must be 2, 4, or 8"):
        QuantizedKVConfig(value_bits=16)
    with pytest.raises(ValueError, match="group_size must be positive"):
        QuantizedKVConfig(group_size=0)
    with pytest.raises(ValueError, match="calibration_tokens must be non-negative"):
        QuantizedKVConfig(calibration_tokens=-1)


def test_kv_functions_validate_before_touching_the_device():
    x = torch.ones(3)
    with pytest.raises(ValueError, match="bits must be 2, 4, or 8"):
        quantize_tensor(x, bits=3)
    with pytest.raises(ValueError, match="bits must be 2, 4, or 8"):
        dequantize_tensor(x, x, x, bits=5, original_shape=(3,))


def test_no_cpu_fallback():
    """CPU tensors are rejected rather than computed on the host."""
    with pytest.raises(ValueError, match="CUDA"):
        quantize_tensor(torch.ones(2, 64), bits=4)
