"""Bounded device waits, exercised without any fault: with the producer
warps stalled (b2f_set_producer_stall, a test control that makes them issue
no copies) and a 20 us wait limit, each kernel family's consumers give up,
skip their work and report B2F_ERR_TIMEOUT -- in the library's sticky status
and, for the plan-driven GEMMs, in the plan's status word -- and the context
stays usable: after the controls are restored the same calls give the
oracle's results."""

import numpy as np
import pytest
import torch

from b200flash import _capi, mx_compat
from b200flash.quantized_kv_cache import decode_attention, quantize_tensor
from oracle import affine
from oracle.fp import round_to

from helpers import assert_close, to_dev, to_np, u32_to_dev

pytestmark = pytest.mark.gpu

B2F_ERR_TIMEOUT = -5


@pytest.fixture
def stalled(dev):
    lib = _capi.lib()
    torch.cuda.synchronize()
    _capi.device_status(clear=True)
    assert lib.b2f_set_wait_limit_ns(20_000) == 0
    assert lib.b2f_set_producer_stall(1) == 0
    try:
        yield
    finally:
        torch.cuda.synchronize()
        lib.b2f_set_producer_stall(0)
        lib.b2f_set_wait_limit_ns(0)
        _capi.device_status(clear=True)


def _experts(rng, E, N, K):
    return affine.quantize(round_to(rng.normal(0, 0.02, (E, N, K)).astype(np.float32), "bf16"), 64, 4)


def _dev3(t, dev):
    return u32_to_dev(t[0], dev), to_dev(t[1], "bf16", dev), to_dev(t[2], "bf16", dev)


def _plan_status(plan):
    return int(plan.workspace[4:8].view(torch.int32).item())


@pytest.mark.parametrize("engine", ["mma", "tc", "tc_sorted"])
def test_expert_gemm_wait_times_out(dev, stalled, engine):
    rng = np.random.default_rng(1)
    E, N, K, T, k = 4, 128, 256, 12, 2
    w = _experts(rng, E, N, K)
    x = to_dev(round_to(rng.standard_normal((T, K)).astype(np.float32), "bf16"), "bf16", dev)
    inds = torch.from_numpy(np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)).to(dev)
    tile = 16 if engine == "mma" else 32
    plan = mx_compat.MoEPlan(inds.reshape(-1), E, tile)
    if engine == "mma":
        mx_compat.gather_qmm_mma_planned(x, plan, *_dev3(w, dev), 64, 4, x_row_div=k)
    elif engine == "tc":
        mx_compat.gather_qmm_tc_planned(x, plan, *_dev3(w, dev), 64, 4, x_row_div=k)
    else:
        xs = mx_compat.moe_gather_rows(x, plan, x_row_div=k)
        mx_compat.sorted_qmm_tc(xs, plan, *_dev3(w, dev), 64, 4)
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == B2F_ERR_TIMEOUT
    assert _plan_status(plan) == B2F_ERR_TIMEOUT


@pytest.mark.parametrize("engine", ["gemv", "tc"])
def test_dense_matmul_wait_times_out(dev, stalled, engine):
    rng = np.random.default_rng(2)
    w = affine.quantize(round_to(rng.normal(0, 0.02, (256, 512)).astype(np.float32), "bf16"), 64, 4)
    x = to_dev(round_to(rng.standard_normal((8, 512)).astype(np.float32), "bf16"), "bf16", dev)
    mx_compat.quantized_matmul(x, *_dev3(w, dev), True, 64, 4, engine=engine)
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == B2F_ERR_TIMEOUT


@pytest.mark.parametrize("bits", [8, 4])
def test_decode_attention_wait_times_out(dev, stalled, bits):
    """The page-ring attention kernels (token-row form for 8-bit d128, head-row
    form for 4-bit): the page copies never come, the page waits give up."""
    rng = np.random.default_rng(3)
    k = round_to(rng.standard_normal((48, 2, 128)).astype(np.float32), "bf16")
    kp, ks, _ = quantize_tensor(to_dev(k, "bf16", dev), bits, 64)
    vp, vs, _ = quantize_tensor(to_dev(k[::-1].copy(), "bf16", dev), bits, 64)

    def head_major(t):
        return t.reshape(3, 16, *t.shape[1:]).permute(0, 2, 1, 3).contiguous()

    q = to_dev(rng.standard_normal((1, 8, 128)).astype(np.float32), "bf16", dev)
    bt = torch.arange(3, dtype=torch.int32, device=dev).reshape(1, 3)
    sl = torch.tensor([40], dtype=torch.int32, device=dev)
    decode_attention(q, head_major(kp), head_major(ks), head_major(vp), head_major(vs), bt, sl, bits, 16, 2)
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == B2F_ERR_TIMEOUT


def test_context_usable_after_timeouts(dev):
    """Runs after the stalled tests in this file: controls restored, the same
    kernels give the oracle's results and no timeout is recorded."""
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == 0
    rng = np.random.default_rng(4)
    E, N, K, T, k = 4, 128, 256, 12, 2
    w = _experts(rng, E, N, K)
    xn = round_to(rng.standard_normal((T, 1, 1, K)).astype(np.float32), "bf16")
    inds = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    for engine in ("mma", "tc", "tc_sorted"):
        out = mx_compat.gather_qmm(to_dev(xn, "bf16", dev), *_dev3(w, dev), rhs_indices=torch.from_numpy(inds).to(dev),
                                   group_size=64, bits=4, engine=engine)
        want = affine.gather_qmm(xn, *w, rhs_indices=inds, group_size=64, bits=4, out_dtype="f32")
        assert_close(to_np(out), want, what=f"gather_qmm {engine} after the timeout tests")
    torch.cuda.synchronize()
    assert _capi.device_status(clear=True) == 0
