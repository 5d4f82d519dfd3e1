"""GPU parity of the rotary embedding + KV scatter kernel (vlc_rope_store_kvcache).

Bit-exact against the reference's own RoPE (fixture rope_3b.npz: nano-vllm's
``apply_rotary_emb`` evaluated eagerly) and against the CPU oracle (oracle/rope.py) at
the BASELINE config 2 / 4 shapes; the fused path of ``Attention.forward`` must give the
same cache and output as rotating first and scattering after.
"""
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import rope as orope

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def mods(cuda_lib):
    from vlcache_b200 import ops
    from vlcache_b200.layers import rotary_embedding as rope
    ops.device_error(reset=True)
    return ops, rope


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def test_rotary_embedding_matches_reference_fixture(mods):
    ops, rope = mods
    f = np.load(GOLDEN / "rope_3b.npz")
    rot = rope.RotaryEmbedding(128, 128, int(f["max_position"]), 1e6).cuda()
    pos = torch.from_numpy(f["positions"]).cuda()
    q_out, k_out = rot(pos, _from_bits(f["q"]).cuda(), _from_bits(f["k"]).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(_bits(q_out), f["q_rot"])
    assert np.array_equal(_bits(k_out), f["k_rot"])
    assert ops.device_error() == 0


@pytest.mark.parametrize("H,Hk,N", [(16, 2, 1123), (28, 4, 10617), (16, 2, 1)])
def test_rope_store_kvcache_matches_oracle(mods, H, Hk, N):
    """Config 2 (3B, 1,123 rows) and config 4 at ratio 1.0 (7B, 10,617 rows): q/k/v are
    views of one qkv row (the reference's split), slots -1 skipped, q rotated in place."""
    ops, rope = mods
    D, NB, BS, max_pos = 128, 64, 256, 32768
    g = torch.Generator().manual_seed(N)
    qkv = torch.randn(N, (H + 2 * Hk) * D, generator=g).mul_(2).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (N,), generator=g, dtype=torch.int64)
    nslots = NB * BS
    slots = torch.randperm(nslots, generator=g)[:N].to(torch.int32)
    slots[::13] = -1
    kc = torch.randn(nslots, Hk, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(nslots, Hk, D, generator=g).to(torch.bfloat16)
    cache = rope.rope_cos_sin_cache(D, max_pos, 1e6)
    q_bits = _bits(qkv[:, :H * D]).reshape(N, H, D)
    k_bits = _bits(qkv[:, H * D:(H + Hk) * D]).reshape(N, Hk, D)
    v_bits = _bits(qkv[:, (H + Hk) * D:]).reshape(N, Hk, D)
    q_ref, kc_ref, vc_ref = orope.rope_store_kvcache(pos.numpy(), q_bits, k_bits, v_bits, cache[:, 0].numpy(),
                                                     _bits(kc).reshape(nslots, -1), _bits(vc).reshape(nslots, -1),
                                                     slots.numpy())
    d_qkv = qkv.cuda()
    q = d_qkv[:, :H * D].view(N, H, D)
    k = d_qkv[:, H * D:(H + Hk) * D].view(N, Hk, D)
    v = d_qkv[:, (H + Hk) * D:].view(N, Hk, D)
    d_kc = kc.cuda().view(NB, BS, Hk, D)   # the paged layout [num_blocks, block_size, Hk, D]
    d_vc = vc.cuda().view(NB, BS, Hk, D)
    out = ops.rope_store_kvcache(pos.cuda(), q, k, v, cache.cuda(), d_kc, d_vc, slots.cuda(), out=q)
    torch.cuda.synchronize()
    assert out.data_ptr() == q.data_ptr()
    assert np.array_equal(_bits(out).reshape(N, H, D), q_ref)
    assert np.array_equal(_bits(d_kc).reshape(nslots, -1), kc_ref)
    assert np.array_equal(_bits(d_vc).reshape(nslots, -1), vc_ref)
    assert ops.device_error() == 0


def test_rope_errors_flagged(mods):
    ops, rope = mods
    cache = rope.rope_cos_sin_cache(128, 64, 1e6).cuda()
    q = torch.randn(3, 4, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(3, 2, 128, device="cuda").to(torch.bfloat16)
    kc = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    pos = torch.tensor([0, 63, 64], device="cuda")     # 64 is past the table
    ops.rope_store_kvcache(pos, q, k, k, cache, kc, vc, torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda"))
    assert ops.device_error(reset=True) == 103
    pos = torch.tensor([0, 1, 2], device="cuda")
    ops.rope_store_kvcache(pos, q, k, k, cache, kc, vc, torch.tensor([0, 8, -1], dtype=torch.int32, device="cuda"))
    assert ops.device_error(reset=True) == 101       # slot 8 of 8
    with pytest.raises(RuntimeError):                  # head_dim 64 is not supported
        ops.rotary_embedding(pos, q[..., :64].contiguous(), k[..., :64].contiguous(),
                             rope.rope_cos_sin_cache(64, 64, 1e6).cuda())


def test_attention_forward_fused_rope_equals_unfused(cuda_lib):
    """Attention.forward(q, k, v, positions, rotary_emb) on un-rotated q/k gives the same
    paged cache and output, bit for bit, as rotating with RotaryEmbedding first."""
    from vlcache_b200 import ops
    from vlcache_b200.engine import kv_cache as kvc
    from vlcache_b200.layers.attention import Attention
    from vlcache_b200.layers.rotary_embedding import get_rope
    from vlcache_b200.utils import context as ctx
    H, Hk, D = 16, 2, 128
    g = torch.Generator().manual_seed(21)
    pre, n_img, suf, R = 20, 700, 30, 70
    n = pre + n_img + suf
    nb = (n + 255) // 256
    bt = torch.randperm(nb + 2, generator=g)[:nb].tolist()
    builder = kvc.WarmPrefillBuilder(H, Hk)
    batch = builder.build([kvc.WarmRequest(n, bt, pre, pre + n_img, R, True)])
    k_cache = torch.randn(nb + 2, 256, Hk, D, generator=g).to(torch.bfloat16).cuda()
    v_cache = torch.randn(nb + 2, 256, Hk, D, generator=g).to(torch.bfloat16).cuda()
    nq = int(batch.cu_seqlens_q[-1])
    qkv = torch.randn(nq, (H + 2 * Hk) * D, generator=g).to(torch.bfloat16).cuda()
    q = qkv[:, :H * D].view(nq, H, D)
    k = qkv[:, H * D:(H + Hk) * D].view(nq, Hk, D)
    v = qkv[:, (H + Hk) * D:].view(nq, Hk, D)
    rot = get_rope(D, D, 32768, 1e6).cuda()
    builder.upload(batch, device="cuda")
    positions = batch.device_tensors["positions"]
    outs = []
    for fused in (False, True):
        attn = Attention(H, D, 1 / math.sqrt(D), Hk)
        attn.k_cache, attn.v_cache = k_cache.clone(), v_cache.clone()
        if fused:
            o = attn(q, k, v, positions=positions, rotary_emb=rot)
        else:
            qr, kr = rot(positions, q, k)
            o = attn(qr, kr, v)
        torch.cuda.synchronize()
        outs.append((o, attn.k_cache, attn.v_cache))
    assert torch.equal(outs[0][1], outs[1][1]) and torch.equal(outs[0][2], outs[1][2])
    assert torch.equal(outs[0][0], outs[1][0])
    assert ops.device_error() == 0
    ctx.reset_context()


def test_attention_forward_decode_fused_rope(cuda_lib):
    """Decode through the fused path: the new token's rotated K lands in its slot and the
    output equals the unfused path (rotate, then scatter and attend) bit for bit."""
    from tests.helpers import make_decode_case
    from vlcache_b200 import ops
    from vlcache_b200.engine import kv_cache as kvc
    from vlcache_b200.layers.attention import Attention
    from vlcache_b200.layers.rotary_embedding import RotaryEmbedding
    from vlcache_b200.utils import context as ctx
    H, Hk, D = 28, 4, 128
    lens = [5000, 257, 1, 3000]
    q, kc, vc, bt, _, scale = make_decode_case(len(lens), H, Hk, lens, seed=23)
    g = torch.Generator().manual_seed(24)
    k_new = torch.randn(len(lens), Hk, D, generator=g).to(torch.bfloat16).cuda()
    v_new = torch.randn(len(lens), Hk, D, generator=g).to(torch.bfloat16).cuda()
    bts = [[int(x) for x in row if x >= 0] for row in bt.tolist()]
    positions = kvc.prepare_decode(lens, bts, device="cuda")
    rot = RotaryEmbedding(D, D, 8192, 1e6).cuda()
    outs = []
    for fused in (False, True):
        attn = Attention(H, D, scale, Hk)
        attn.k_cache, attn.v_cache = kc.cuda(), vc.cuda()
        if fused:
            o = attn(q.cuda(), k_new, v_new, positions=positions, rotary_emb=rot)
        else:
            qr, kr = rot(positions, q.cuda(), k_new)
            o = attn(qr, kr, v_new)
        torch.cuda.synchronize()
        outs.append((o, attn.k_cache, attn.v_cache))
    assert outs[1][0].shape == (len(lens), 1, H, D)
    assert torch.equal(outs[0][1], outs[1][1]) and torch.equal(outs[0][2], outs[1][2])
    assert torch.equal(outs[0][0], outs[1][0])
    assert ops.device_error() == 0
    ctx.reset_context()
