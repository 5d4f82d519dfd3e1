"""GPU parity of the vision tower's varlen attention (head_dim 80, non-causal).

The reference runs ``flash_attn_varlen_func(q, k, v, cu_seqlens, cu_seqlens, ...,
causal=False)`` in every Qwen2.5-VL vision block (nanovllm/models/qwen2_5_vl.py:202-211):
window attention over ~64-patch windows (qwen2_5_vl.py:392-435) and full attention over
the image in the full-attention blocks.  ``layers.vision_attention.varlen_attention`` runs
the tcgen05 kernel with a non-causal plan; it is compared with the fp32 oracle
(``oracle.attention.varlen_attention``) and with flash-attn 2.8.3 on the same inputs,
within max-abs 2e-2 / mean-abs 2e-3.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu

ATT_MAX, ATT_MEAN = 2e-2, 2e-3


def _window_lens(grid_h: int, grid_w: int, merge: int = 2, window_merged: int = 4):
    """Patch counts of the vision windows of a merged grid, in raster order of windows:
    window_merged x window_merged merged tokens (merge^2 patches each), smaller at the
    right and bottom borders (the layout of qwen2_5_vl.py:392-435's get_window_index)."""
    lens = []
    for r0 in range(0, grid_h, window_merged):
        for c0 in range(0, grid_w, window_merged):
            lens.append(min(window_merged, grid_h - r0) * min(window_merged, grid_w - c0) * merge * merge)
    return lens


def _cu(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def _check(margins, what, a, b):
    d = (a.float().cpu() - b.float().cpu()).abs()
    mx, mean = float(d.max()), float(d.mean())
    margins(what, mx, mean)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (what, mx, mean)


def _qkv(n, H, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn(n, 3, H, d, generator=g, device="cuda").to(torch.bfloat16)
    return qkv[:, 0], qkv[:, 1], qkv[:, 2]          # token stride 3 * H * d, like a fused QKV split


@pytest.mark.parametrize("d", [80, 128])
def test_window_attention_1080p(cuda_lib, margins, d):
    """The window layout of a 1920x1080 image (39 x 69 merged grid, 10,764 patches, ragged
    border windows), 16 heads: kernel vs oracle on every row and vs flash-attn."""
    from vlcache_b200.layers.vision_attention import varlen_attention
    lens = _window_lens(39, 69)
    cu = _cu(lens)
    n = int(cu[-1])
    assert n == 39 * 69 * 4
    q, k, v = _qkv(n, 16, d, seed=d)
    scale = 1.0 / math.sqrt(d)
    cu_d = torch.from_numpy(cu).cuda()
    out = varlen_attention(q, k, v, cu_d, cu_d, max(lens), max(lens), scale, causal=False, cu_seqlens_q_host=cu,
                           cu_seqlens_k_host=cu)
    torch.cuda.synchronize()
    from vlcache_b200 import ops
    assert ops.device_error() == 0
    ref = oatt.varlen_attention(q.cpu(), k.cpu(), v.cpu(), cu, cu, scale, causal=False)
    _check(margins, f"vision windows d={d} kernel vs oracle", out, ref)
    fa = pytest.importorskip("flash_attn")
    fo = fa.flash_attn_varlen_func(q, k, v, cu_d, cu_d, max(lens), max(lens), softmax_scale=scale, causal=False)
    _check(margins, f"vision windows d={d} kernel vs flash-attn", out, fo)


def test_full_attention_1080p(cuda_lib, margins):
    """A full-attention vision block over a 1080p image (10,764 patches, non-causal), 16
    heads of 80: kernel vs flash-attn on every row, vs the oracle on 96 seeded rows."""
    from vlcache_b200.layers.vision_attention import varlen_attention
    n, H, d = 39 * 69 * 4, 16, 80
    q, k, v = _qkv(n, H, d, seed=5)
    cu = np.array([0, n], np.int32)
    cu_d = torch.from_numpy(cu).cuda()
    scale = 1.0 / math.sqrt(d)
    out = varlen_attention(q, k, v, cu_d, cu_d, n, n, scale, cu_seqlens_q_host=cu, cu_seqlens_k_host=cu)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(3).choice(n, 96, replace=False))
    sub = oatt._attend(q.cpu().float()[rows], k.cpu().float(), v.cpu().float(), torch.full((96,), n - 1), scale)
    _check(margins, "vision full attention kernel vs oracle (96 rows)", out[torch.from_numpy(rows).cuda()], sub)
    fa = pytest.importorskip("flash_attn")
    fo = fa.flash_attn_varlen_func(q, k, v, cu_d, cu_d, n, n, softmax_scale=scale, causal=False)
    _check(margins, "vision full attention kernel vs flash-attn", out, fo)


def test_causal_contiguous_head_dim_80_and_clipped_stores(cuda_lib, margins):
    """Causal varlen attention at head_dim 80 (contiguous K/V, split tiles included), into
    an output whose rows are wider than H x 80: the columns past each row's heads stay
    untouched, so every store stops at the real head width."""
    from vlcache_b200 import ops
    from vlcache_b200.layers.vision_attention import varlen_attention
    lens_q, lens_k = [300, 48, 7, 129], [300, 6000, 7, 900]
    cq, ck = _cu(lens_q), _cu(lens_k)
    H, d = 16, 80
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(int(cq[-1]), H, d, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(int(ck[-1]), H, d, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(int(ck[-1]), H, d, generator=g, device="cuda").to(torch.bfloat16)
    wide = torch.zeros(int(cq[-1]), H * d + 64, dtype=torch.bfloat16, device="cuda")
    out = wide[:, :H * d].view(int(cq[-1]), H, d)
    scale = 1.0 / math.sqrt(d)
    varlen_attention(q, k, v, torch.from_numpy(cq).cuda(), torch.from_numpy(ck).cuda(), causal=True,
                     softmax_scale=scale, cu_seqlens_q_host=cq, cu_seqlens_k_host=ck, out=out)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert int(wide[:, H * d:].abs().sum()) == 0
    ref = oatt.varlen_attention(q.cpu(), k.cpu(), v.cpu(), cq, ck, scale, causal=True)
    _check(margins, "causal contiguous d=80 kernel vs oracle", out, ref)


@pytest.mark.parametrize("H,Hk,d,maxlen", [(16, 16, 80, 128), (16, 2, 128, 16)])
def test_packed_short_sequences(cuda_lib, margins, H, Hk, d, maxlen):
    """Non-causal self-attention of short sequences of random lengths 1..maxlen (whole
    sequences packed several to a tile, block-diagonal mask), GQA included: kernel vs oracle
    on every row and vs flash-attn."""
    from vlcache_b200.layers.vision_attention import varlen_attention
    rng = np.random.default_rng(d + maxlen)
    lens = rng.integers(1, maxlen + 1, size=300).tolist()
    cu = _cu(lens)
    n = int(cu[-1])
    g = torch.Generator(device="cuda").manual_seed(17)
    q = torch.randn(n, H, d, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(n, Hk, d, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(n, Hk, d, generator=g, device="cuda").to(torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    cu_d = torch.from_numpy(cu).cuda()
    out = varlen_attention(q, k, v, cu_d, cu_d, max(lens), max(lens), scale, cu_seqlens_q_host=cu,
                           cu_seqlens_k_host=cu)
    torch.cuda.synchronize()
    from vlcache_b200 import ops
    assert ops.device_error() == 0
    ref = oatt.varlen_attention(q.cpu(), k.cpu(), v.cpu(), cu, cu, scale, causal=False)
    _check(margins, f"packed sequences H={H} Hk={Hk} d={d} kernel vs oracle", out, ref)
    fa = pytest.importorskip("flash_attn")
    fo = fa.flash_attn_varlen_func(q, k, v, cu_d, cu_d, max(lens), max(lens), softmax_scale=scale, causal=False)
    _check(margins, f"packed sequences H={H} Hk={Hk} d={d} kernel vs flash-attn", out, fo)
