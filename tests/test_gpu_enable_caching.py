"""enable_caching (vllm_integration.py:41-111) on a small PyTorch MoE model
shaped like mlx-lm's (model.model.layers[i].mlp with gate, top_k,
switch_mlp.{gate,up,down}_proj, shared_expert, shared_expert_gate): the
swapped projections and the skip-fallback forward vs the oracle."""

import numpy as np
import pytest
import torch

from b200flash.expert_streaming import CachedSwitchLinear
from b200flash.vllm_integration import enable_caching
from oracle import affine, moe
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


class QSwitchLinear(torch.nn.Module):
    def __init__(self, t, dev):
        super().__init__()
        self.weight, self.scales, self.biases = u32_to_dev(t[0], dev), to_dev(t[1], "bf16", dev), to_dev(t[2], "bf16", dev)
        self.group_size, self.bits = 64, 4


class QLinear(QSwitchLinear):
    pass


class SwitchGLU(torch.nn.Module):
    def __init__(self, g, u, d, dev):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = (QSwitchLinear(t, dev) for t in (g, u, d))


class SharedMLP(torch.nn.Module):
    def __init__(self, g, u, d, dev):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = (QLinear(t, dev) for t in (g, u, d))


class MoEBlock(torch.nn.Module):
    def __init__(self, wr, experts, k, dev, shared=None, shared_gate=None):
        super().__init__()
        E, H = wr.shape
        self.gate = torch.nn.Linear(H, E, bias=False, device=dev, dtype=torch.bfloat16)
        self.gate.weight.data.copy_(to_dev(wr, "bf16", dev))
        self.top_k = k
        self.switch_mlp = SwitchGLU(*experts, dev)
        if shared is not None:
            self.shared_expert = SharedMLP(*shared, dev)
            self.shared_expert_gate = torch.nn.Linear(H, 1, bias=False, device=dev, dtype=torch.bfloat16)
            self.shared_expert_gate.weight.data.copy_(to_dev(shared_gate, "bf16", dev))

    def forward(self, x):
        raise RuntimeError("the unpatched forward is the host framework's, not under test")


class Layer(torch.nn.Module):
    def __init__(self, mlp):
        super().__init__()
        self.mlp = mlp


class Inner(torch.nn.Module):
    def __init__(self, layers):
        super().__init__()
        self.layers = torch.nn.ModuleList(layers)


class Model(torch.nn.Module):
    def __init__(self, layers):
        super().__init__()
        self.model = Inner(layers)


def _q(rng, shape):
    return affine.quantize(round_to(rng.normal(0, 0.02, shape).astype(np.float32), "bf16"), 64, 4)


@pytest.mark.parametrize("skip", [2.0, 1e-3])
def test_enable_caching_skip_fallback_forward(dev, skip):
    rng = np.random.default_rng(int(skip * 7))
    E, H, I, Is, k, T = 16, 512, 256, 384, 4, 20
    layers, refs = [], []
    for li in range(2):
        ex = tuple(_q(rng, shp) for shp in ((E, I, H), (E, I, H), (E, H, I)))
        wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
        sh = tuple(_q(rng, shp) for shp in ((Is, H), (Is, H), (H, Is))) if li == 1 else None
        sg = round_to(rng.normal(0, 0.05, (1, H)).astype(np.float32), "bf16") if li == 1 else None
        layers.append(Layer(MoEBlock(wr, ex, k, dev, sh, sg)))
        refs.append((wr, ex, sh, sg))
    model = Model(layers)
    state = enable_caching(model, capacity_per_layer=64, adaptive_skip_threshold=skip)
    assert len(state.caches) == 2 and state.total_cached() == 2 * E and state.avg_coverage() == 1.0
    assert isinstance(model.model.layers[0].mlp.switch_mlp.gate_proj, CachedSwitchLinear)
    x = round_to(rng.standard_normal((T, H)).astype(np.float32), "bf16")
    for li, (wr, ex, sh, sg) in enumerate(refs):
        out = model.model.layers[li].mlp(to_dev(x, "bf16", dev).reshape(2, T // 2, H))
        assert tuple(out.shape) == (2, T // 2, H)
        oi, os_ = moe.route(x, wr.T, k, renorm=True, skip_threshold=skip)
        want, _, _ = moe.expert_mlp(x, oi, os_, *ex)
        if sh is not None:
            want = want + moe.shared_expert(x, *sh, sg)
        assert_close(to_np(out).reshape(T, H), want, what=f"enable_caching layer {li} skip {skip}")
    if skip >= 1:
        assert (os_ == 0).any(), "the LExI threshold never fired"
    state.update()
    assert state.stats()[0]["tokens"] == 1


def test_enable_caching_without_skip_swaps_projections(dev):
    """adaptive_skip_threshold 0: only the projections are swapped; each is
    gather_qmm over the cached stack (CachedSwitchLinear.__call__)."""
    rng = np.random.default_rng(4)
    E, H, I, k, T = 8, 256, 128, 2, 6
    ex = tuple(_q(rng, shp) for shp in ((E, I, H), (E, I, H), (E, H, I)))
    wr = round_to(rng.normal(0, 0.05, (E, H)).astype(np.float32), "bf16")
    model = Model([Layer(MoEBlock(wr, ex, k, dev))])
    enable_caching(model)
    sw = model.model.layers[0].mlp.switch_mlp
    x = round_to(rng.standard_normal((T, 1, 1, H)).astype(np.float32), "bf16")
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    out = sw.up_proj(to_dev(x, "bf16", dev), torch.from_numpy(inds).to(dev))
    want = affine.gather_qmm(x, *ex[1], rhs_indices=inds, group_size=64, bits=4, out_dtype="f32")
    assert_close(to_np(out), want, what="CachedSwitchLinear up_proj")
