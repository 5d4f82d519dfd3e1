"""GPU tests of the public, reference-shaped API (Attention.forward, set_context, the warm
metadata builder, the all-layer image-KV shift) and of the remaining BASELINE configs,
all against the CPU oracle.  Tolerances as in test_gpu_kernels.py."""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import mrope as omr
from tests.helpers import attn_errors, make_decode_case, make_warm_case

pytestmark = pytest.mark.gpu
ATT_MAX, ATT_MEAN = 2e-2, 2e-3


@pytest.fixture(scope="module")
def api(cuda_lib):
    from vlcache_b200 import ops
    from vlcache_b200.engine import kv_cache as kvc
    from vlcache_b200.layers.attention import Attention
    from vlcache_b200.utils import context as ctx
    ops.device_error(reset=True)
    return ops, kvc, Attention, ctx


@pytest.mark.parametrize("gated", [False, True])
def test_attention_forward_warm_prefill(api, gated):
    """Warm request through the drop-in layer: recomputed K/V are scattered by the layer,
    then the recomputed rows attend over the paged cache (reused image rows included).
    gated: the layer first waits for its Context.kv_ready event (recorded on a side stream)."""
    ops, kvc, Attention, ctx = api
    H, Hk, D = 16, 2, 128
    g = torch.Generator().manual_seed(11)
    pre, n_img, suf, R = 20, 700, 30, 70
    n = pre + n_img + suf
    nb = (n + 255) // 256
    bt = torch.randperm(nb + 2, generator=g)[:nb].tolist()
    req = kvc.WarmRequest(n, bt, pre, pre + n_img, R, True)
    builder = kvc.WarmPrefillBuilder(H, Hk)
    batch = builder.build([req])
    k_cache = torch.randn(nb + 2, 256, Hk, D, generator=g).to(torch.bfloat16)
    v_cache = torch.randn(nb + 2, 256, Hk, D, generator=g).to(torch.bfloat16)
    nq = int(batch.cu_seqlens_q[-1])
    qkv = torch.randn(nq, (H + 2 * Hk) * D, generator=g).to(torch.bfloat16)
    q = qkv[:, :H * D].view(nq, H, D)
    k = qkv[:, H * D:(H + Hk) * D].view(nq, Hk, D)
    v = qkv[:, (H + Hk) * D:].view(nq, Hk, D)
    # oracle: scatter on CPU, then attention
    kc_ref, vc_ref = k_cache.clone(), v_cache.clone()
    slots = torch.from_numpy(batch.slot_mapping).long()
    kc_ref.view(-1, Hk, D)[slots] = k
    vc_ref.view(-1, Hk, D)[slots] = v
    ref = oatt.prefill_attention(q, kc_ref, vc_ref, batch.block_tables, batch.cu_seqlens_q, batch.cu_seqlens_k,
                                 1 / math.sqrt(D))
    attn = Attention(H, D, 1 / math.sqrt(D), Hk)
    attn.k_cache, attn.v_cache = k_cache.cuda(), v_cache.cuda()
    builder.upload(batch, device="cuda")
    if gated:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        ev = torch.cuda.Event()
        with torch.cuda.stream(side):
            torch.cuda._sleep(1000)
            ev.record(side)
        ctx.get_context().kv_ready = [ev]
        attn.layer_id = 0
    out = attn(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    assert torch.equal(attn.k_cache.cpu(), kc_ref) and torch.equal(attn.v_cache.cpu(), vc_ref)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)
    ctx.reset_context()


def test_attention_forward_cold_prefill_contiguous(api):
    """Cold prefill (no block tables): the layer attends over the in-flight K/V."""
    ops, kvc, Attention, ctx = api
    H, Hk, D = 28, 4, 128
    g = torch.Generator().manual_seed(12)
    lens = [300, 1, 517]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    tot = int(cu[-1])
    qkv = torch.randn(tot, (H + 2 * Hk) * D, generator=g).to(torch.bfloat16)
    q = qkv[:, :H * D].view(tot, H, D)
    k = qkv[:, H * D:(H + Hk) * D].view(tot, Hk, D)
    v = qkv[:, (H + Hk) * D:].view(tot, Hk, D)
    ref = torch.zeros(tot, H, D)
    for b in range(len(lens)):
        s, e = cu[b], cu[b + 1]
        ref[s:e] = oatt._attend(q[s:e].float(), k[s:e].float(), v[s:e].float(), torch.arange(e - s), 1 / math.sqrt(D))
    attn = Attention(H, D, 1 / math.sqrt(D), Hk)   # no KV cache attached: nothing is scattered
    cq = torch.from_numpy(cu).cuda()
    ctx.set_context(True, cq, cq, max(lens), max(lens), None, None, None)
    out = attn(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)
    ctx.reset_context()


def test_attention_forward_decode(api):
    ops, kvc, Attention, ctx = api
    H, Hk, D = 28, 4, 128
    lens = [5000, 257, 1, 3000]   # lengths after appending the new token
    q, kc, vc, bt, _, scale = make_decode_case(len(lens), H, Hk, lens, seed=13)
    g = torch.Generator().manual_seed(14)
    k_new = torch.randn(len(lens), Hk, D, generator=g).to(torch.bfloat16)
    v_new = torch.randn(len(lens), Hk, D, generator=g).to(torch.bfloat16)
    bts = [[int(x) for x in row if x >= 0] for row in bt.tolist()]
    positions = kvc.prepare_decode(lens, bts, device="cuda")
    assert positions.tolist() == [n - 1 for n in lens]
    c = ctx.get_context()
    kc_ref, vc_ref = kc.clone(), vc.clone()
    slots = c.slot_mapping.cpu().long()
    kc_ref.view(-1, Hk, D)[slots] = k_new
    vc_ref.view(-1, Hk, D)[slots] = v_new
    ref = oatt.decode_attention(q, kc_ref, vc_ref, bt, torch.tensor(lens), scale)
    attn = Attention(H, D, scale, Hk)
    attn.k_cache, attn.v_cache = kc.cuda(), vc.cuda()
    out = attn(q.cuda(), k_new.cuda(), v_new.cuda())
    torch.cuda.synchronize()
    assert out.shape == (len(lens), 1, H, D)
    mx, mean = attn_errors(out[:, 0], ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)
    ctx.reset_context()


def test_decode_graph_replay_with_new_lengths(api):
    """The decode launch is capture-safe: a captured graph replays correctly after the
    context lengths (device data) change, as nano-vllm's decode graphs do."""
    ops, kvc, Attention, ctx = api
    H, Hk = 16, 2
    lens = [2000, 600, 4000]
    q, kc, vc, bt, ctxl, scale = make_decode_case(3, H, Hk, lens, seed=15)
    qd, kd, vd, btd, ld = q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), ctxl.cuda()
    max_len = bt.shape[1] * 256
    out = torch.empty_like(qd)
    ws = torch.empty(max(1, ops.decode_workspace_bytes(3, H, Hk, max_len)), dtype=torch.uint8, device="cuda")
    ops.decode_attention(qd, kd, vd, btd, ld, max_len, scale, out, ws)   # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.decode_attention(qd, kd, vd, btd, ld, max_len, scale, out, ws)
    for new in ([2000, 600, 4000], [1999, 1, 3500]):
        ld.copy_(torch.tensor(new, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        ref = oatt.decode_attention(q, kc, vc, bt, torch.tensor(new), scale)
        mx, mean = attn_errors(out, ref)
        assert mx <= ATT_MAX and mean <= ATT_MEAN, (new, mx, mean)


def test_copy_image_kv_all_layers_with_shift(api):
    """Reused image rows of every layer move to the new request's pages, K re-rotated by the
    M-RoPE delta, V verbatim; other rows untouched."""
    ops, kvc, Attention, ctx = api
    L, NB, Hk, D = 4, 10, 2, 128
    g = torch.Generator().manual_seed(16)
    kv = torch.randn(2, L, NB, 256, Hk, D, generator=g).to(torch.bfloat16)
    old_bt, new_bt = [0, 1, 2, 3], [7, 4, 9, 5]
    old_slots, new_slots = kvc.image_reuse_slots(30, 30 + 700, 70, new_bt, 10, old_bt)
    from vlcache_b200.layers.rotary_embedding import image_position_delta
    delta = image_position_delta(10, 30)
    assert delta == (20, 20, 20)
    kvd = kv.cuda()
    kvc.copy_image_kv(kvd, old_slots, new_slots, delta)
    torch.cuda.synchronize()
    got = kvd.cpu()
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    for layer in range(L):
        src_k = bits(kv[0, layer]).reshape(-1, Hk, D)[old_slots]
        exp_k = omr.shift_rows(src_k, delta)
        got_k = bits(got[0, layer]).reshape(-1, Hk, D)[new_slots]
        diff = np.abs(omr.bf16_bits_to_f32(got_k) - omr.bf16_bits_to_f32(exp_k))
        assert np.all(diff <= np.abs(omr.bf16_bits_to_f32(exp_k)) * 2.0 ** -7 + 1e-30)
        assert np.array_equal(bits(got[1, layer]).reshape(-1, Hk * D)[new_slots],
                              bits(kv[1, layer]).reshape(-1, Hk * D)[old_slots])
        untouched = np.setdiff1d(np.arange(NB * 256), new_slots)
        assert np.array_equal(bits(got[0, layer]).reshape(-1, Hk * D)[untouched],
                              bits(kv[0, layer]).reshape(-1, Hk * D)[untouched])


def test_copy_image_kv_per_layer_matches_one_launch(api):
    """The per-layer variant (one launch per layer on a side stream, one event per layer)
    leaves the cache bit-identical to the all-layers launch."""
    ops, kvc, Attention, ctx = api
    L, NB, Hk, D = 3, 10, 2, 128
    g = torch.Generator().manual_seed(17)
    kv = torch.randn(2, L, NB, 256, Hk, D, generator=g).to(torch.bfloat16)
    old_slots, new_slots = kvc.image_reuse_slots(30, 30 + 700, 70, [7, 4, 9, 5], 10, [0, 1, 2, 3])
    delta = (20, 20, 20)
    a, b = kv.cuda(), kv.cuda()
    kvc.copy_image_kv(a, old_slots, new_slots, delta)
    side = torch.cuda.Stream()
    src = torch.from_numpy(old_slots).cuda()
    dst = torch.from_numpy(new_slots).cuda()
    ready = kvc.copy_image_kv_per_layer(b, src, dst, delta, side)
    assert len(ready) == L
    for ev in ready:
        torch.cuda.current_stream().wait_event(ev)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ops.device_error() == 0


def test_prefill_cfg3_style_batch(api):
    """BASELINE config 3 shape (per request: 2,691-token image, ratio 0.05, prefix U[0,512],
    suffix U[16,128]) for a batch of 12 warm requests in one launch."""
    ops, *_ = api
    rng = np.random.default_rng(3)
    n_img, R = 39 * 69, math.ceil(0.05 * 39 * 69)
    specs = [(int(p), n_img, int(s), R) for p, s in zip(rng.integers(0, 513, 12), rng.integers(16, 129, 12))]
    case = make_warm_case(specs, 16, 2, device="cuda", seed=17)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, 16, 2, device="cuda")
    out = ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_cfg4_ratio_002_7b(api):
    """BASELINE config 4 (Qwen2.5-VL-7B heads), recompute ratio 0.02 (211 rows) of a 4K image."""
    ops, *_ = api
    case = make_warm_case([(20, 10549, 48, 211)], 28, 4, device="cuda", seed=18)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, 28, 4, device="cuda")
    out = ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


# ------------------------------------------------------------------ device metadata builder
def _golden_reqs(name):
    from pathlib import Path
    from vlcache_b200.engine import kv_cache as kvc
    g = dict(np.load(Path(__file__).resolve().parent / "golden" / f"metadata_{name}.npz"))
    reqs = []
    for i, (n, s, e, R, partial) in enumerate(g["requests"]):
        bt = [int(x) for x in g["request_block_tables"][i] if x >= 0]
        reqs.append(kvc.WarmRequest(int(n), bt, int(s) if s >= 0 else None, int(e) if e >= 0 else None, int(R),
                                    bool(partial)))
    reuse = [kvc.ImageReuse(i, int(g["cold_img_start"]), [int(x) for x in g["cold_block_table"]])
             for i, r in enumerate(reqs) if r.partial]
    return g, reqs, reuse


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "mixed"])
def test_device_metadata_matches_reference_fixtures(api, name):
    """The device builder reproduces, bit for bit, the metadata the reference's own
    prepare_prefill / _do_image_kv_copy produced for these batches (golden fixtures)."""
    ops, kvc, Attention, ctx = api
    g, reqs, reuse = _golden_reqs(name)
    b = kvc.WarmPrefillBuilder(16, 2).build_device(reqs, reuse, device="cuda", install=False)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    t = b.device_tensors
    assert np.array_equal(b.cu_seqlens_q, g["cu_seqlens_q"]) and np.array_equal(b.cu_seqlens_k, g["cu_seqlens_k"])
    assert np.array_equal(t["positions"].cpu().numpy(), g["positions"])
    assert np.array_equal(t["slot_mapping"].cpu().numpy(), g["slot_mapping"])
    assert np.array_equal(t["block_tables"].cpu().numpy(), g["block_tables"])
    assert list(b.logit_indices) == list(g["logit_indices"])
    assert np.array_equal(t["reuse_src"].cpu().numpy(), g["old_slots"])
    assert np.array_equal(t["reuse_dst"].cpu().numpy(), g["new_slots"])


def test_device_metadata_matches_host_builder_cfg3_batch(api):
    """64 warm requests of BASELINE config 3 shape (plus two cold ones): device and host
    builders agree on every array, and the reuse slots equal image_reuse_slots."""
    ops, kvc, Attention, ctx = api
    rng = np.random.default_rng(31)
    n_img, R = 39 * 69, kvc.recompute_count(0.05, 39 * 69)
    reqs, reuse, next_page = [], [], 0
    for i in range(66):
        pre, suf = int(rng.integers(0, 513)), int(rng.integers(16, 129))
        n = pre + n_img + suf if i < 64 else int(rng.integers(1, 3000))
        nb = (n + 255) // 256
        bt = list(range(next_page, next_page + nb))
        next_page += nb
        if i < 64:
            reqs.append(kvc.WarmRequest(n, bt, pre, pre + n_img, R, True))
            reuse.append(kvc.ImageReuse(i, 7, list(range(900000, 900000 + 12))))
        else:
            reqs.append(kvc.WarmRequest(n, bt))
    builder = kvc.WarmPrefillBuilder(16, 2)
    host = builder.build(reqs)
    dev = builder.build_device(reqs, reuse, device="cuda", install=False)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    t = dev.device_tensors
    assert np.array_equal(t["positions"].cpu().numpy(), host.positions)
    assert np.array_equal(t["slot_mapping"].cpu().numpy(), host.slot_mapping)
    assert np.array_equal(t["block_tables"].cpu().numpy(), host.block_tables)
    assert np.array_equal(dev.cu_seqlens_q, host.cu_seqlens_q) and np.array_equal(dev.cu_seqlens_k, host.cu_seqlens_k)
    src = np.concatenate([kvc.image_reuse_slots(reqs[i].img_start, reqs[i].img_end, R, reqs[i].block_table, 7,
                                                list(range(900000, 900012)))[0] for i in range(64)])
    dst = np.concatenate([kvc.image_reuse_slots(reqs[i].img_start, reqs[i].img_end, R, reqs[i].block_table, 7,
                                                list(range(900000, 900012)))[1] for i in range(64)])
    assert np.array_equal(t["reuse_src"].cpu().numpy(), src)
    assert np.array_equal(t["reuse_dst"].cpu().numpy(), dst)


def test_device_metadata_flags_short_block_table(api):
    """A block table too short for a request's positions: device error 102, slot -1."""
    ops, kvc, Attention, ctx = api
    ops.device_error(reset=True)
    reqs = [kvc.WarmRequest(700, [3, 5])]          # 700 tokens need 3 pages of 256
    b = kvc.WarmPrefillBuilder(16, 2).build_device(reqs, device="cuda", install=False)
    torch.cuda.synchronize()
    assert ops.device_error(reset=True) == 102
    s = b.device_tensors["slot_mapping"].cpu().numpy()
    assert np.array_equal(s[:512], np.concatenate([np.arange(768, 1024), np.arange(1280, 1536)]))
    assert np.all(s[512:] == -1)


def test_allocate_kv_cache_sized_from_free_memory(cuda_lib):
    """allocate_kv_cache(num_blocks=None) sizes the pool with the reference's rule
    (model_runner.py:130-151) and hands each Attention module its layer's K/V views and
    layer_id (model_runner.py:152-158)."""
    from torch import nn

    from vlcache_b200.engine import kv_cache as kvc
    from vlcache_b200.layers.attention import Attention

    class Toy(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList([nn.ModuleDict({"attn": Attention(16, 128, 0.088, 2)}) for _ in range(4)])

    model = Toy()
    free, total = torch.cuda.mem_get_info()
    stats = torch.cuda.memory_stats()
    # the rule subtracts torch's peak allocation (minus what is still allocated), which the
    # tests run before this one raise: leave about 3 GiB to the caches on top of it
    slack = stats.get("allocated_bytes.all.peak", 0) - stats.get("allocated_bytes.all.current", 0)
    util = (total - free + slack + 3 * 2 ** 30) / total
    kv = kvc.allocate_kv_cache(model, 4, None, 2, hidden_size=2048, gpu_memory_utilization=util,
                               encoder_cache_ratio=0.2, device="cuda")
    b = kv.budget
    assert kv.shape == (2, 4, b.num_kvcache_blocks, 256, 2, 128) and b.num_encoder_blocks > 0
    assert 0.5 * 2 ** 30 < b.num_kvcache_blocks * b.kv_block_bytes <= 3 * 2 ** 30
    for i, layer in enumerate(model.layers):
        a = layer["attn"]
        assert a.layer_id == i
        assert a.k_cache.data_ptr() == kv[0, i].data_ptr() and a.v_cache.data_ptr() == kv[1, i].data_ptr()
        assert a.k_cache.shape == (b.num_kvcache_blocks, 256, 2, 128)
