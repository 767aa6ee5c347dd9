"""The allocation-free decode attention entry point, called through the C ABI.

``b2f_qkv_decode_attn_noalloc`` serves callers that cannot allocate device
memory when they run decode attention -- a C / cgo / JNI host with no device
allocator of its own, or a process whose GPU memory is already owned by
another framework's pool.  Its split-K scratch is a fixed 4 MiB array inside
the library.  This test checks it against the workspace-taking
``b2f_qkv_decode_attn`` on two calls in a row (the second with other inputs,
so stale scratch contents from the first call would show), and that a
request larger than the array is refused without a launch.

The file name sorts last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process.
"""

import pytest
import torch

from b200flash import _capi
from b200flash.quantized_kv_cache import packed_len

from helpers import assert_close

pytestmark = pytest.mark.gpu

HQ, HKV, D, PAGE = 32, 8, 128, 64


def _case(dev, seed, B, lens, bits):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    pl = packed_len(D, bits, 64)
    pages_per = [(n + PAGE - 1) // PAGE for n in lens]
    total = sum(pages_per)
    maxp = max(pages_per)
    kp = torch.randint(0, 256, (total, HKV, PAGE, pl), dtype=torch.uint8, device=dev, generator=g)
    vp = torch.randint(0, 256, (total, HKV, PAGE, pl), dtype=torch.uint8, device=dev, generator=g)
    if bits == 8:
        kp.clamp_(max=254)
        vp.clamp_(max=254)
    else:
        kp.copy_(((kp % 15) << 4) | (kp // 16 % 15))
        vp.copy_(((vp % 15) << 4) | (vp // 16 % 15))
    ks = torch.rand(total, HKV, PAGE, D // 64, device=dev, generator=g) * 0.05 + 0.01
    vs = torch.rand(total, HKV, PAGE, D // 64, device=dev, generator=g) * 0.05 + 0.01
    perm = torch.randperm(total, device=dev, generator=g).to(torch.int32)
    bt = torch.zeros(B, maxp, dtype=torch.int32, device=dev)
    cur = 0
    for b, n in enumerate(pages_per):
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    q = torch.randn(B, HQ, D, device=dev, generator=g).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, kp, ks, vp, vs, bt, sl


def _args(q, kp, ks, vp, vs, bt, sl, bits, n_splits):
    B = q.shape[0]
    return (q.data_ptr(), kp.data_ptr(), ks.data_ptr(), vp.data_ptr(), vs.data_ptr(), bt.data_ptr(), bt.shape[1],
            sl.data_ptr(), B, HQ, HKV, D, PAGE, PAGE, 1, bits, 64, D ** -0.5, n_splits)


def _with_workspace(case, bits, n_splits, dev):
    q = case[0]
    out = torch.empty_like(q)
    nb = int(_capi.lib().b2f_qkv_decode_attn_workspace_bytes(q.shape[0], HQ, D, n_splits))
    ws = torch.empty(max(nb, 16), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _capi.lib().b2f_qkv_decode_attn(*_args(*case, bits, n_splits), ws.data_ptr(), nb, out.data_ptr(), stream)
    assert rc == 0, _capi.status_text(rc)
    return out


def _no_alloc(case, bits, n_splits, dev):
    out = torch.empty_like(case[0])
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _capi.lib().b2f_qkv_decode_attn_noalloc(*_args(*case, bits, n_splits), out.data_ptr(), stream)
    assert rc == 0, _capi.status_text(rc)
    return out


def test_noalloc_matches_workspace_entry_point_twice(dev):
    # first call: 8-bit cache, 6 context splits
    a = _case(dev, 1, 6, [1, 77, 700, 2048, 3000, 64], 8)
    want1 = _with_workspace(a, 8, 6, dev)
    got1 = _no_alloc(a, 8, 6, dev)
    # second call right after, different sizes/bits: stale scratch must not matter
    b = _case(dev, 2, 3, [5000, 130, 2], 4)
    want2 = _with_workspace(b, 4, 9, dev)
    got2 = _no_alloc(b, 4, 9, dev)
    torch.cuda.synchronize()
    for got, want, tag in ((got1, want1, "first"), (got2, want2, "second")):
        assert torch.isfinite(got.float()).all(), tag
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), what=f"noalloc {tag} call")


def test_noalloc_rejects_requests_beyond_the_scratch_size(dev):
    # B*Hq*splits*(D+2)*4 bytes > 4 MiB: refused before any launch
    a = _case(dev, 3, 2, [64, 64], 8)
    out = torch.empty_like(a[0])
    big_B = 64
    args = list(_args(*a, 8, 64))
    args[8] = big_B  # claims 64 sequences x 64 splits
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _capi.lib().b2f_qkv_decode_attn_noalloc(*args, out.data_ptr(), stream)
    assert rc == _capi.B2F_ERR_WORKSPACE
    torch.cuda.synchronize()
