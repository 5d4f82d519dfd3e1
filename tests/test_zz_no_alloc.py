"""The decode entry point that allocates nothing (vlc_decode_attn_noalloc).

It serves callers that may not allocate device memory (fixed memory budgets, no
cudaMalloc after start-up): its split-K partials live in a library-owned 8 MiB device
array instead of a caller workspace.  This file is collected last so that a run that
stops at its first failure has already run every other test; it also passes alone.
The checks: two calls in a row with different inputs through the C ABI give the same
result as the workspace entry point and as the fp32 CPU oracle, within the attention
tolerance of the other tests; and once the library's device code is loaded, a call leaves
the device's free memory unchanged (it allocates nothing).
"""
import ctypes

import pytest
import torch

from oracle import attention as oatt
from tests.helpers import make_decode_case

pytestmark = pytest.mark.gpu

ATT_MAX, ATT_MEAN = 2e-2, 2e-3


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _noalloc(lib, q, kc, vc, bt, ctx, max_len, scale, out):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.vlc_decode_attn_noalloc(_p(q), q.stride(0), q.shape[0], q.shape[1], _p(kc), _p(vc),
                                       kc.shape[0] * kc.shape[1], kc.shape[2], kc.shape[3], _p(bt), bt.stride(0),
                                       kc.shape[1], _p(ctx), max_len, scale, _p(out), out.stride(0), stream)


def test_noalloc_decode_matches_workspace_decode_twice(cuda_lib):
    from vlcache_b200 import ops
    assert cuda_lib.vlc_decode_noalloc_scratch_bytes() == 8 << 20
    for seed, lens in ((21, [3000, 64, 10700, 257, 5000, 1]), (22, [9000, 700, 4097, 2711])):
        q, kc, vc, bt, ctx, scale = make_decode_case(len(lens), 28, 4, lens, device="cuda", seed=seed)
        max_len = max(lens)
        need = ops.decode_workspace_bytes(len(lens), 28, 4, max_len)
        assert 0 < need <= cuda_lib.vlc_decode_noalloc_scratch_bytes()
        ref = ops.decode_attention(q, kc, vc, bt, ctx, max_len, scale)
        out = torch.full_like(ref, float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        assert _noalloc(cuda_lib, q, kc, vc, bt, ctx, max_len, scale, out) == 0
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        assert ops.device_error() == 0
        if seed != 21:   # the first call may load the library's device code (and its array)
            assert free_after == free_before, (free_before, free_after)
        d = (out.float() - ref.float()).abs()
        assert torch.isfinite(out).all()
        assert float(d.max()) <= ATT_MAX and float(d.mean()) <= ATT_MEAN
        orc = oatt.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), ctx.cpu(), scale)
        d = (out.float().cpu() - orc).abs()
        assert float(d.max()) <= ATT_MAX and float(d.mean()) <= ATT_MEAN


def test_noalloc_decode_rejects_requests_beyond_scratch(cuda_lib):
    from vlcache_b200 import ops
    # 256 sequences x 28 heads x up to 64k keys needs far more than 8 MiB of partials.
    n, max_len = 256, 65536
    assert ops.decode_workspace_bytes(n, 28, 4, max_len) > cuda_lib.vlc_decode_noalloc_scratch_bytes()
    q = torch.zeros(n, 28, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 256, 4, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(n, 1, dtype=torch.int32, device="cuda")
    ctx = torch.ones(n, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    assert _noalloc(cuda_lib, q, kc, kc, bt, ctx, max_len, 0.1, out) == 6   # VLC_ERR_WORKSPACE, nothing launched
    assert int(out.abs().sum()) == 0
