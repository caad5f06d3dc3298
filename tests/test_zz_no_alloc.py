"""The allocation-free attention entry point (b2_attention_decode_noalloc).

For callers that cannot call cudaMalloc -- a serving process whose HBM is
already fully reserved by its own pools, or a per-token path that cannot
afford the device-wide synchronisation an allocation can cause -- the library
offers the decode attention with its split partials kept in a fixed 2 MiB
in-library device array.  These tests call it through the C ABI and compare
it with the allocating entry point on two calls in a row (the second call
must not be affected by what the first left in the shared array), check the
size limit, and check that repeated calls leave the device's free memory
unchanged.  The file is named to be collected last.
"""
import numpy as np
import pytest

import b2decode

pytestmark = pytest.mark.gpu

TOL = 1e-4  # relative L2, as for the allocating attention entry point


def _inputs(torch, batch, nh, nkv, hd, ctx, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((batch, nh * hd), device="cuda", generator=g)
    k = torch.randn((batch, ctx, nkv * hd), device="cuda", generator=g).half()
    v = torch.randn((batch, ctx, nkv * hd), device="cuda", generator=g).half()
    return q, k, v


def _call(fn, q, k, v, out, batch, nh, nkv, hd, ctx):
    fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, nh, nkv, hd, ctx)


@pytest.mark.parametrize("batch,nh,nkv,hd,ctx", [(1, 32, 8, 128, 4096), (8, 32, 8, 128, 4096), (2, 14, 2, 64, 300)])
def test_noalloc_matches_allocating_entry_point(built_lib, batch, nh, nkv, hd, ctx):
    import torch
    for seed in (11, 12):  # two calls in a row
        q, k, v = _inputs(torch, batch, nh, nkv, hd, ctx, seed)
        ref = torch.empty((batch, nh * hd), device="cuda")
        got = torch.full((batch, nh * hd), float("nan"), device="cuda")
        _call(b2decode.attention_decode, q, k, v, ref, batch, nh, nkv, hd, ctx)
        _call(b2decode.attention_decode_noalloc, q, k, v, got, batch, nh, nkv, hd, ctx)
        torch.cuda.synchronize()
        a, b = got.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
        assert np.isfinite(a).all()
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(built_lib):
    import torch
    q = torch.zeros(8, device="cuda")
    kv = torch.zeros(8, dtype=torch.float16, device="cuda")
    out = torch.zeros(8, device="cuda")
    with pytest.raises(b2decode.B2Error) as e:
        # 2048 * 32 * (128 + 2) floats > 524288
        b2decode.attention_decode_noalloc(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), 2048, 32, 8,
                                          128, 16)
    assert e.value.code == -8
    assert "allocation-free scratch" in str(e.value)


def test_noalloc_leaves_free_memory_unchanged(built_lib):
    import torch
    batch, nh, nkv, hd, ctx = 2, 32, 8, 128, 2048
    q, k, v = _inputs(torch, batch, nh, nkv, hd, ctx, 5)
    out = torch.empty((batch, nh * hd), device="cuda")
    _call(b2decode.attention_decode_noalloc, q, k, v, out, batch, nh, nkv, hd, ctx)  # first call: set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        _call(b2decode.attention_decode_noalloc, q, k, v, out, batch, nh, nkv, hd, ctx)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
