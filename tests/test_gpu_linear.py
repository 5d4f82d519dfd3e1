"""GPU parity of the recomputed rows' linear layers (tcgen05 GEMM, vlc_linear*).

* ``vlc_linear`` against an fp32 torch reference of F.linear: every output within one
  bf16 ulp of the fp32 result (relative 2^-7, plus 1e-2 of the output's RMS for
  cancellation), at the BASELINE shapes (Qwen2.5-VL-3B / 7B projections of the 1,123
  recomputed cfg2 rows) and at ragged M / N tails.
* ``vlc_linear_silu_mul`` against silu(g) * u evaluated in fp32 from the bf16-rounded
  gate / up outputs (SiluAndMul of nanovllm/layers/activation.py on F.linear's output).
* ``vlc_qkv_rope_store_kvcache`` bit-exact against the same GEMM (vlc_linear with the
  bias) followed by the RoPE + KV-scatter kernel (whose bit-exactness against the
  reference's RotaryEmbedding is pinned by tests/test_gpu_rope.py), and within
  tolerance of the fp32 reference path; cache rows of skipped (-1) slots untouched.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[1, 2, 3, 4, 0], ids=["single_sm", "cta_pair", "single_sm_128", "single_sm_224", "auto"])
def kernel_mode(request, cuda_lib):
    """Run a test on each GEMM configuration: single-SM 128 x 256 tiles, CTA pairs
    (cta_group::2, 256 x 256), single-SM 128 x 128 and 128 x 224 (the plain epilogue; the
    others fall back), and the automatic choice."""
    from vlcache_b200 import ops
    ops.set_linear_kernel(request.param)
    yield request.param
    ops.set_linear_kernel(0)


def _ref_linear(x, w, b=None):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y


# Relative bounds.  A plain linear rounds once (fp32 accumulator -> bf16): one ulp, 2^-7.
# The fused epilogues round the linear's output to bf16 first (as the reference, whose
# F.linear returns bf16) and then compute on it: where the GEMM's accumulation order puts
# an accumulator next to a bf16 rounding boundary, that input can differ from the fp32
# reference's rounding by one ulp, and two such inputs (gate and up, or x1 and x2 of a
# rotation) plus the output rounding compound to about 3 ulps: 2^-5.
ONE_ULP, FUSED = 2.0 ** -7, 2.0 ** -5


def _assert_close_ulp(out, ref, what, margins, bound=ONE_ULP):
    ref = ref.float()
    d = (out.float() - ref).abs()
    rms = float(ref.pow(2).mean().sqrt())
    rel = d / (ref.abs() + 1e-2 * rms)
    margins(f"{what} (rel {float(rel.max()):.2e} / {bound:.2e})", float(d.max()), float(d.mean()),
            tol_max=float("inf"), tol_mean=float("inf"))
    assert float(rel.max()) <= bound, (what, float(rel.max()))


@pytest.mark.parametrize("m,n,k,bias", [
    (1123, 2560, 2048, True),     # 3B qkv_proj (cfg2 rows)
    (1123, 2048, 2048, False),    # 3B o_proj
    (1123, 2048, 11008, False),   # 3B down_proj
    (1123, 4608, 3584, True),     # 7B qkv_proj
    (1, 256, 512, False),
    (129, 136, 64, True),         # N tail inside a 32-column chunk, M tail
    (300, 520, 200, False),       # K not a multiple of 64
])
def test_linear_matches_fp32(kernel_mode, margins, m, n, k, bias):
    from vlcache_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
    b = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16) if bias else None
    out = ops.linear(x, w, b)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    _assert_close_ulp(out, _ref_linear(x, w, b), f"linear {m}x{n}x{k}", margins)


@pytest.mark.parametrize("m,n,k", [(1123, 2048, 11008), (1123, 3584, 18944), (200, 512, 4096), (1, 256, 8192)])
def test_linear_stream_k(cuda_lib, margins, m, n, k):
    """The stream-K split (K-block ranges over one CTA per SM, partial tiles fixed up by
    the CTA that completes them) against fp32, against whole-tile launches, run to run
    bit-identical, and the workspace's tickets left at zero for the next launch."""
    from vlcache_b200 import ops
    ops.set_linear_kernel(1)   # stream-K belongs to the single-SM kernel
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
    b = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
    sk = ops.linear(x, w, b, stream_k=True)
    sk2 = ops.linear(x, w, b, stream_k=True)
    whole = ops.linear(x, w, b, stream_k=False)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = _ref_linear(x, w, b)
    _assert_close_ulp(sk, ref, f"linear stream-K {m}x{n}x{k}", margins)
    _assert_close_ulp(whole, ref, f"linear whole tiles {m}x{n}x{k}", margins)
    assert torch.equal(sk.view(torch.int16), sk2.view(torch.int16))
    ws, _ = ops.linear_workspace(ops.LINEAR, m, n, k, x.device)
    tiles = -(-m // 128) * -(-n // 256)
    off = 2 * ops.num_sms() * 128 * 256 * 4   # the tickets follow the per-SM partial slots
    assert int(ws[off:off + 4 * tiles].view(torch.int32).abs().sum()) == 0
    ops.set_linear_kernel(0)


def test_linear_strided_input_and_output(kernel_mode, margins):
    """x and out as column slices of wider buffers (row strides != widths)."""
    from vlcache_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(7)
    xb = torch.randn(200, 1024, generator=g, device="cuda").to(torch.bfloat16)
    x = xb[:, 64:64 + 512]
    w = (torch.randn(384, 512, generator=g, device="cuda") / 23.0).to(torch.bfloat16)
    ob = torch.zeros(200, 1000, dtype=torch.bfloat16, device="cuda")
    out = ob[:, 8:8 + 384]
    ops.linear(x, w, out=out)
    torch.cuda.synchronize()
    _assert_close_ulp(out, _ref_linear(x, w), "linear strided", margins)
    assert int(ob[:, :8].abs().sum()) == 0 and int(ob[:, 392:].abs().sum()) == 0


@pytest.mark.parametrize("m,inter,k", [(1123, 11008, 2048), (1123, 18944, 3584), (77, 200, 128)])
def test_linear_silu_mul(kernel_mode, margins, m, inter, k):
    from vlcache_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + inter)
    x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(2 * inter, k, generator=g, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
    out = ops.linear_silu_mul(x, w)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    gu = _ref_linear(x, w).to(torch.bfloat16).float()
    gate, up = gu[:, :inter], gu[:, inter:]
    ref = gate / (1.0 + torch.exp(-gate)) * up
    _assert_close_ulp(out, ref, f"silu_mul {m}x{inter}x{k}", margins, FUSED)


@pytest.mark.parametrize("H,Hk,hidden", [(16, 2, 2048), (28, 4, 3584)])
def test_qkv_rope_store_bit_exact_vs_unfused(kernel_mode, margins, H, Hk, hidden):
    from oracle import rope as orope
    from vlcache_b200 import ops
    from vlcache_b200.layers.rotary_embedding import rope_cos_sin_cache
    D, m, max_pos = 128, 1123, 16384
    g = torch.Generator(device="cuda").manual_seed(H)
    x = torch.randn(m, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((H + 2 * Hk) * D, hidden, generator=g, device="cuda") / math.sqrt(hidden)).to(torch.bfloat16)
    b = torch.randn((H + 2 * Hk) * D, generator=g, device="cuda").to(torch.bfloat16)
    table = rope_cos_sin_cache(D, max_pos, 1e6).to("cuda")
    pos = torch.randint(0, max_pos, (m,), generator=g, device="cuda")
    num_slots = 2048
    slots = torch.randperm(num_slots, generator=g, device="cuda")[:m].to(torch.int32)
    slots[::17] = -1
    # the paged layout [num_blocks, 256, Hk, D] (store_kvcache's stride contract)
    kc0 = torch.randn(num_slots // 256, 256, Hk, D, generator=g, device="cuda").to(torch.bfloat16)
    vc0 = torch.randn(num_slots // 256, 256, Hk, D, generator=g, device="cuda").to(torch.bfloat16)
    # fused
    kc, vc = kc0.clone(), vc0.clone()
    q = ops.qkv_rope_store_kvcache(x, w, b, pos, table, kc, vc, slots, H, Hk)
    # unfused: the same GEMM, then the RoPE + scatter kernel
    qkv = ops.linear(x, w, b)
    kc2, vc2 = kc0.clone(), vc0.clone()
    q2 = ops.rope_store_kvcache(pos, qkv[:, :H * D].view(m, H, D), qkv[:, H * D:(H + Hk) * D].view(m, Hk, D),
                                qkv[:, (H + Hk) * D:].view(m, Hk, D), table, kc2, vc2, slots)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(q.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(kc.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc.view(torch.int16), vc2.view(torch.int16))
    # rows whose slot is -1 (and slots nobody maps) keep their old contents
    used = torch.zeros(num_slots, dtype=torch.bool, device="cuda")
    used[slots[slots >= 0].long()] = True
    assert torch.equal(kc.view(num_slots, -1)[~used].view(torch.int16), kc0.view(num_slots, -1)[~used].view(torch.int16))
    # against the fp32 reference path (F.linear in fp32 -> bf16, oracle RoPE)
    ref_qkv = _ref_linear(x, w, b).to(torch.bfloat16)
    bits = lambda t: t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    sl = slots.cpu().numpy()
    q_ref, kc_ref, vc_ref = orope.rope_store_kvcache(
        pos.cpu().numpy(), bits(ref_qkv[:, :H * D]).reshape(m, H, D),
        bits(ref_qkv[:, H * D:(H + Hk) * D]).reshape(m, Hk, D), bits(ref_qkv[:, (H + Hk) * D:]).reshape(m, Hk, D),
        table.cpu().numpy(), bits(kc0).reshape(num_slots, -1), bits(vc0).reshape(num_slots, -1), sl)
    as_f = lambda u: torch.from_numpy(u.astype(np.uint16).view(np.int16)).view(torch.bfloat16).float()  # noqa: E731
    rq = ref_qkv.float().cpu()
    _assert_rope_close(q.cpu(), as_f(q_ref).view(m, H, D), rq[:, :H * D].reshape(m, H, D), f"qkv_rope q (H={H})",
                       margins)
    kv_rows = torch.from_numpy(sl)
    keep = kv_rows >= 0
    k_pre = rq[:, H * D:(H + Hk) * D].reshape(m, Hk, D)[keep]
    _assert_rope_close(kc.view(num_slots, Hk, D).cpu()[kv_rows[keep].long()],
                       as_f(kc_ref).view(num_slots, Hk, D)[kv_rows[keep].long()], k_pre, f"qkv_rope k cache (H={H})",
                       margins)
    _assert_close_ulp(vc.float().cpu().view(num_slots, Hk, D), as_f(vc_ref).view(num_slots, Hk, D),
                      f"qkv_rope v cache (H={H})", margins)


def test_qkv_rope_store_errors_match_unfused(kernel_mode):
    """Rows with an out-of-range rotary position or cache slot: the fused kernel records
    the same device error as the RoPE + scatter kernel and leaves the same outputs (a bad
    position skips the row's q and k, a bad slot its k and v), bit for bit."""
    from vlcache_b200 import ops
    from vlcache_b200.layers.rotary_embedding import rope_cos_sin_cache
    D, H, Hk, hidden, m, max_pos, num_slots = 128, 16, 2, 256, 300, 512, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(m, hidden, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((H + 2 * Hk) * D, hidden, generator=g, device="cuda") / 16).to(torch.bfloat16)
    b = torch.randn((H + 2 * Hk) * D, generator=g, device="cuda").to(torch.bfloat16)
    table = rope_cos_sin_cache(D, max_pos, 1e6).to("cuda")
    kc0 = torch.randn(num_slots // 256, 256, Hk, D, generator=g, device="cuda").to(torch.bfloat16)
    qkv = ops.linear(x, w, b)
    for bad, code in (("pos", 103), ("slot", 101)):
        pos = torch.randint(0, max_pos, (m,), generator=g, device="cuda")
        slots = torch.randperm(num_slots, generator=g, device="cuda")[:m].to(torch.int32)
        if bad == "pos":
            pos[[5, 130, 299]] = max_pos
        else:
            slots[[7, 200]] = num_slots
        outs = []
        for fused in (True, False):
            kc, vc = kc0.clone(), kc0.clone()
            q = torch.full((m, H, D), 7.0, dtype=torch.bfloat16, device="cuda")
            ops.device_error(reset=True)
            if fused:
                ops.qkv_rope_store_kvcache(x, w, b, pos, table, kc, vc, slots, H, Hk, q_out=q)
            else:
                ops.rope_store_kvcache(pos, qkv[:, :H * D].view(m, H, D), qkv[:, H * D:(H + Hk) * D].view(m, Hk, D),
                                       qkv[:, (H + Hk) * D:].view(m, Hk, D), table, kc, vc, slots, out=q)
            torch.cuda.synchronize()
            assert ops.device_error(reset=True) == code, (bad, fused)
            outs.append((q, kc, vc))
        for a, c in zip(*outs):
            assert torch.equal(a.view(torch.int16), c.view(torch.int16)), bad


def _assert_rope_close(out, ref, x_pre, what, margins):
    """A rotation y1 = x1 c - x2 s, y2 = x2 c + x1 s of bf16 inputs that may each differ by
    one ulp from the fp32 reference's rounding: |err| <= 2^-7 (|x1| + |x2|) of the pair's
    reference inputs, plus the output's own rounding 2^-8 |y|.  (Bounded by the inputs,
    not the output: where x1 c ~ x2 s the output is near zero and an input ulp is not.)"""
    out, ref, x_pre = out.float(), ref.float(), x_pre.float()
    half = x_pre.shape[-1] // 2
    pair = x_pre.abs() + torch.cat([x_pre[..., half:], x_pre[..., :half]], -1).abs()
    d = (out - ref).abs()
    ratio = d / (2.0 ** -7 * pair + 2.0 ** -8 * ref.abs() + 1e-6)
    margins(f"{what} (bound use {float(ratio.max()):.2f})", float(d.max()), float(d.mean()),
            tol_max=float("inf"), tol_mean=float("inf"))
    assert float(ratio.max()) <= 1.0, (what, float(ratio.max()))


def test_linear_layers_dropin(cuda_lib):
    """The layer classes load weights like the reference's (packed q/k/v and gate/up
    shards) and their forwards equal the ops they wrap."""
    from vlcache_b200 import ops
    from vlcache_b200.layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
    g = torch.Generator().manual_seed(5)
    qkv = QKVParallelLinear(256, 128, 4, 2, bias=True)
    parts = {s: torch.randn(n * 128, 256, generator=g) / 16 for s, n in (("q", 4), ("k", 2), ("v", 2))}
    for s, t in parts.items():
        qkv.weight.weight_loader(qkv.weight, t, s)
        qkv.bias.weight_loader(qkv.bias, torch.randn(t.shape[0], generator=g), s)
    assert torch.equal(qkv.weight.data, torch.cat([parts["q"], parts["k"], parts["v"]]))
    gu = MergedColumnParallelLinear(256, [384, 384])
    gate, up = torch.randn(384, 256, generator=g) / 16, torch.randn(384, 256, generator=g) / 16
    gu.weight.weight_loader(gu.weight, gate, 0)
    gu.weight.weight_loader(gu.weight, up, 1)
    assert torch.equal(gu.weight.data, torch.cat([gate, up]))
    down = RowParallelLinear(384, 256)
    down.weight.weight_loader(down.weight, torch.randn(256, 384, generator=g) / 20)
    for mod in (qkv, gu, down):
        mod.to(device="cuda", dtype=torch.bfloat16)
    x = torch.randn(3, 33, 256, generator=g).to(device="cuda", dtype=torch.bfloat16)
    y = qkv(x)
    assert y.shape == (3, 33, 1024)
    assert torch.equal(y.view(-1, 1024), ops.linear(x.view(-1, 256), qkv.weight, qkv.bias))
    h = gu.forward_silu_mul(x)
    assert h.shape == (3, 33, 384)
    assert torch.equal(h.view(-1, 384), ops.linear_silu_mul(x.view(-1, 256), gu.weight))
    z = down(h)
    assert z.shape == (3, 33, 256)
    torch.cuda.synchronize()
