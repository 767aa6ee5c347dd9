"""Shared helpers for the GPU parity tests (numpy <-> torch, tolerances)."""

import numpy as np
import torch

# matmul / attention outputs in bf16: |got - want| <= ATOL + RTOL*|want|
RTOL = 1e-2
ATOL = 2e-2

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def to_dev(a, dtype, dev):
    """float32 numpy array (values exact in ``dtype``) -> device tensor of ``dtype``."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(TORCH_DT[dtype])


def to_np(t):
    if t.dtype == torch.uint32:
        return t.cpu().view(torch.int32).numpy().view(np.uint32)
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def u32_to_dev(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).to(dev).view(torch.uint32)


def assert_close(got, want, rtol=RTOL, atol=ATOL, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(int(np.argmax(err - bound)), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} outside tolerance; worst at {i}: "
                             f"got {got[i]!r} want {want[i]!r} (max abs err {err.max():.3e})")
