"""GPU parity for the smaller ops: Q4_0 dequant-GEMV (vs the C restatement
of the Metal shader), the kernels/ops.py drop-ins (SwiGLU, moe_dispatch),
4-bit -> 2-bit requantization (bit-exact vs the reference's own NumPy
outputs and the oracle), 2-bit dequantization, sensitivity fake
quantization, and the QuantizedLinear / LayerQuantizer mirror."""

import numpy as np
import pytest
import torch

from b200flash import kernels, mixed_precision
from b200flash.layer_quantization import (LayerQuantConfig, LayerSensitivityProfile, QuantizedLinear,
                                          apply_layer_quantization, fake_quantize_sym)
from oracle import affine, mixed, q4_0, sensitivity
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,gs,nvec", [(1, 32, 32, 1), (37, 96, 32, 1), (4096, 4096, 32, 1),
                                        (300, 6144, 64, 3), (129, 2080, 32, 2)])
def test_q4_0_gemv_matches_shader_restatement(dev, M, N, gs, nvec):
    rng = np.random.default_rng(M + N)
    w = rng.integers(0, 256, (M, N // 2), dtype=np.uint8)
    s = (rng.random((M, N // gs)) * 0.02 + 0.001).astype(np.float16)
    x = rng.standard_normal((nvec, N)).astype(np.float32)
    y = kernels.flash_dequant_gemv_q4(torch.from_numpy(w).to(dev), torch.from_numpy(s).to(dev),
                                      torch.from_numpy(x if nvec > 1 else x[0]).to(dev), gs)
    got = to_np(y).reshape(nvec, M)
    for b in range(nvec):
        want = q4_0.gemv(w, s, x[b], gs)
        # fp32 sums in another order: relative to the scale of the terms
        scale = np.abs(q4_0.gemv_numpy(np.full_like(w, 0xFF), s, np.abs(x[b]), gs)) + 1e-6
        assert np.all(np.abs(got[b] - want) <= 1e-4 * scale + 1e-5), (b, np.abs(got[b] - want).max())


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_swiglu(dev, dtype):
    rng = np.random.default_rng(1)
    g = round_to(rng.standard_normal(4099).astype(np.float32) * 3, dtype)
    u = round_to(rng.standard_normal(4099).astype(np.float32), dtype)
    out = kernels.swiglu(to_dev(g, dtype, dev), to_dev(u, dtype, dev))
    gd, ud = g.astype(np.float64), u.astype(np.float64)
    want = gd / (1 + np.exp(-gd)) * ud
    tol = {"bf16": 1e-2, "f16": 2e-3, "f32": 1e-5}[dtype]
    assert_close(to_np(out), want, rtol=tol, atol=tol, what=f"swiglu {dtype}")


def test_moe_dispatch_matches_reference_numpy(dev, golden):
    z = golden("moe_dispatch.npz")
    for case in sorted({k.split("/")[0] for k in z.files}):
        eo, ids, w, want = (z[f"{case}/{n}"] for n in ("outputs", "ids", "weights", "result"))
        got = kernels.moe_dispatch(torch.from_numpy(eo.astype(np.float32)).to(dev),
                                   torch.from_numpy(ids.astype(np.int32)).to(dev),
                                   torch.from_numpy(w.astype(np.float32)).to(dev))
        assert_close(to_np(got), want, rtol=1e-5, atol=1e-5, what=f"moe_dispatch {case}")


def test_moe_dispatch_batched_bf16(dev):
    rng = np.random.default_rng(4)
    T, E, H, k = 5, 8, 264, 3
    eo = round_to(rng.standard_normal((T, E, H)).astype(np.float32), "bf16")
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    got = kernels.moe_dispatch(to_dev(eo, "bf16", dev), torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev))
    want = np.stack([(eo[t][ids[t]] * w[t][:, None]).sum(0) for t in range(T)])
    assert_close(to_np(got), want, what="moe_dispatch batched")


def test_requant_4to2_bit_exact_vs_reference(dev, golden):
    z = golden("mixed2bit.npz")
    for case in sorted({k.split("/")[0] for k in z.files}):
        wq, s, b = z[f"{case}/wq"], z[f"{case}/scales"], z[f"{case}/biases"]
        p, s2, b2, meta = mixed_precision.requantize_4bit_to_2bit(u32_to_dev(wq, dev), torch.from_numpy(s).to(dev),
                                                                 torch.from_numpy(b).to(dev))
        assert np.array_equal(to_np(p), z[f"{case}/packed2"]), case
        assert np.array_equal(to_np(s2).astype(np.float16).view(np.uint16),
                              z[f"{case}/scales2"].view(np.uint16)), case
        assert np.array_equal(to_np(b2).astype(np.float16).view(np.uint16),
                              z[f"{case}/biases2"].view(np.uint16)), case
        n = wq.shape[1] * 8
        d = mixed_precision.dequantize_2bit(p, s2, b2, n)
        assert np.array_equal(to_np(d).view(np.uint32), z[f"{case}/deq2"].view(np.uint32)), case
        assert meta["packed_shape"] == z[f"{case}/packed2"].shape


@pytest.mark.parametrize("rows,K,gs,dtype", [(96, 2048, 64, "bf16"), (33, 768, 128, "f16"), (7, 512, 32, "f32"),
                                             (5, 1024, 256, "bf16"), (3, 2048, 1024, "bf16")])
def test_requant_4to2_bit_exact_vs_oracle(dev, rows, K, gs, dtype):
    rng = np.random.default_rng(rows * K)
    w = round_to(rng.normal(0, 0.02, (rows, K)).astype(np.float32), "bf16")
    w[1, :gs] = 0.0  # constant group: range floor 1e-10
    wq, s, b = affine.quantize(w, gs, 4, dtype)
    p, s2, b2, _ = mixed_precision.requantize_4bit_to_2bit(u32_to_dev(wq, dev), to_dev(s, dtype, dev),
                                                           to_dev(b, dtype, dev))
    wp, ws, wb = mixed.requantize_4bit_to_2bit(wq, s, b)
    assert np.array_equal(to_np(p), wp)
    assert np.array_equal(to_np(s2).astype(np.float16), ws)
    assert np.array_equal(to_np(b2).astype(np.float16), wb)


@pytest.mark.parametrize("dtype,bits", [("bf16", 4), ("bf16", 8), ("f16", 4), ("f32", 8)])
def test_fake_quant_sym_matches_oracle(dev, dtype, bits):
    rng = np.random.default_rng(bits)
    w = round_to(rng.normal(0, 0.05, (300, 257)).astype(np.float32), dtype)
    out, amax = fake_quantize_sym(to_dev(w, dtype, dev), bits)
    want, wamax = sensitivity.fake_quantize_sym(w, bits, dtype)
    assert float(amax.item()) == float(wamax)
    assert np.array_equal(to_np(out).view(np.uint32), want.view(np.uint32))
    zero, z_amax = fake_quantize_sym(torch.zeros(64, dtype=torch.float32, device=dev), bits)
    assert float(z_amax.item()) == 0.0 and not torch.any(zero).item()


class _Block(torch.nn.Module):
    def __init__(self, H, I):
        super().__init__()
        self.mlp = torch.nn.Module()
        self.mlp.gate_proj = torch.nn.Linear(H, I, bias=False)
        self.mlp.up_proj = torch.nn.Linear(H, I, bias=False)
        self.mlp.down_proj = torch.nn.Linear(I, H, bias=False)

    def forward(self, x):
        m = self.mlp
        return m.down_proj(torch.nn.functional.silu(m.gate_proj(x)) * m.up_proj(x))


class _Model(torch.nn.Module):
    def __init__(self, n, H, I):
        super().__init__()
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList([_Block(H, I) for _ in range(n)])


def test_quantized_linear_from_linear(dev):
    torch.manual_seed(0)
    lin = torch.nn.Linear(512, 200, bias=True).to(dev)
    ql = QuantizedLinear.from_linear(lin, group_size=64, bits=4)
    wq, s, b = affine.quantize(round_to(lin.weight.detach().float().cpu().numpy(), "bf16"), 64, 4)
    assert np.array_equal(to_np(ql.weight), wq)
    for M in (3, 96):
        x = torch.randn(M, 512, device=dev).to(torch.bfloat16)
        want = affine.quantized_matmul(to_np(x), wq, s, b, True, 64, 4) + to_np(lin.bias.detach().to(torch.bfloat16))
        assert_close(to_np(ql(x)), want, what=f"QuantizedLinear M={M}")


def test_layer_quantizer_and_sensitivity(dev):
    torch.manual_seed(1)
    model = _Model(6, 256, 128).to(dev)
    x = torch.randn(4, 256, device=dev)
    prof = LayerSensitivityProfile(6)
    scores = prof.measure_sensitivity(model, x)
    assert len(scores) == 6 and all(sc > 0 for sc in scores)
    # weights restored after profiling
    assert all(isinstance(l.mlp.gate_proj, torch.nn.Linear) and l.mlp.gate_proj.weight.dtype == torch.float32
               for l in model.model.layers)
    pm = prof.get_precision_map(LayerQuantConfig())
    assert sorted(set(pm.values())) <= [4, 8] and list(pm.values()).count(8) >= 1
    assert LayerSensitivityProfile.default_precision_map(6) == {0: 8, 1: 8, 2: 4, 3: 4, 4: 8, 5: 8}
    res = apply_layer_quantization(model)
    assert res["stats"]["linears_quantized"] == 18
    assert isinstance(model.model.layers[0].mlp.down_proj, QuantizedLinear)
    assert model.model.layers[0].mlp.down_proj.bits == 8 and model.model.layers[3].mlp.down_proj.bits == 4
    assert res["memory"]["effective_bits"] == pytest.approx((4 * 8 + 2 * 4) / 6)
    y = model.model.layers[2](x.to(torch.bfloat16))
    assert torch.isfinite(y.float()).all()
