"""GPU parity of the four hot-path kernels against the CPU oracle (called through the C ABI).

Tolerances: slot scatter bit-exact; bf16 attention outputs
max-abs <= 2e-2 and mean-abs <= 2e-3 against the fp32 oracle; the M-RoPE shift
within 1 bf16 ulp of the oracle's identical fp32 rotation.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import mrope as omr
from tests.helpers import (QWEN_3B, QWEN_7B, attn_errors, cfg2_spec, make_decode_case, make_warm_case,
                           poison_unused_slots)

pytestmark = pytest.mark.gpu

ATT_MAX, ATT_MEAN = 2e-2, 2e-3


@pytest.fixture(scope="module")
def ops(cuda_lib):
    from vlcache_b200 import ops as _ops
    _ops.device_error(reset=True)
    return _ops


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# ------------------------------------------------------------------ store_kvcache
@pytest.mark.parametrize("hk", [2, 4])
def test_store_kvcache_bit_exact(ops, hk):
    g = torch.Generator().manual_seed(1)
    H, N, NB, BS = 8 * hk, 1123, 64, 256
    qkv = torch.randn(N, (H + 2 * hk) * 128, generator=g).to(torch.bfloat16).cuda()
    q, k, v = qkv.split([H * 128, hk * 128, hk * 128], dim=-1)
    k = k.view(N, hk, 128)
    v = v.view(N, hk, 128)
    kc = torch.zeros(NB, BS, hk, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.randperm(NB * BS, generator=g)[:N].to(torch.int32)
    slots[::17] = -1
    slots_d = slots.cuda()
    ops.store_kvcache(k, v, kc, vc, slots_d)
    torch.cuda.synchronize()
    ref_k = torch.zeros(NB * BS, hk * 128, dtype=torch.bfloat16)
    ref_v = torch.zeros_like(ref_k)
    keep = slots >= 0
    ref_k[slots[keep].long()] = k.cpu().reshape(N, -1)[keep]
    ref_v[slots[keep].long()] = v.cpu().reshape(N, -1)[keep]
    assert np.array_equal(_bits(kc.view(-1, hk * 128)), _bits(ref_k))
    assert np.array_equal(_bits(vc.view(-1, hk * 128)), _bits(ref_v))
    assert ops.device_error() == 0


def test_store_kvcache_bad_slot_flagged(ops):
    k = torch.randn(4, 2, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, 1, 512, -1], dtype=torch.int32, device="cuda")  # 512 is out of range
    ops.store_kvcache(k, k, kc, vc, slots)
    assert ops.device_error(reset=True) == 101
    assert torch.equal(kc.view(-1, 256)[0], k[0].reshape(-1))


def test_bounded_wait_gives_up_and_context_stays_usable(ops):
    """Every kernel's barrier waits are bounded: a wait on a barrier nothing completes gives
    up after the limit (~1 ms here), records TIMEOUT + role, and the next launches run."""
    import ctypes
    from vlcache_b200._lib import lib
    L = lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.vlc_selftest_bounded_wait(2_000_000, 1, stream) == 0     # completed barrier: no error
    assert ops.device_error(reset=True) == 0
    assert L.vlc_selftest_bounded_wait(2_000_000, 0, stream) == 0     # never completed: gives up
    assert ops.device_error(reset=True) == 110 + 31
    k = torch.randn(4, 2, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16, device="cuda")
    ops.store_kvcache(k, k, kc, torch.zeros_like(kc), torch.tensor([3, 0, 7, 9], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(kc.view(-1, 256)[3], k[0].reshape(-1))


# ------------------------------------------------------------------ M-RoPE shift
@pytest.mark.parametrize("hk,delta", [(2, (16, 16, 16)), (4, (37, 5, -3))])
def test_mrope_shift_matches_oracle(ops, hk, delta):
    g = torch.Generator().manual_seed(2)
    NB, BS, n = 12, 256, 1500
    kc = torch.randn(NB, BS, hk, 128, generator=g).to(torch.bfloat16)
    vc = torch.randn(NB, BS, hk, 128, generator=g).to(torch.bfloat16)
    perm = torch.randperm(NB * BS, generator=g)
    src, dst = perm[:n].to(torch.int32), perm[n:2 * n].to(torch.int32)
    kd, vd = kc.cuda(), vc.cuda()
    ops.mrope_shift(kd, vd, src.cuda(), dst.cuda(), delta)
    torch.cuda.synchronize()
    kb = _bits(kc).reshape(NB * BS, hk, 128)
    exp = omr.shift_rows(kb[src.numpy()], delta)
    got = _bits(kd).reshape(NB * BS, hk, 128)[dst.numpy()]
    diff = np.abs(omr.bf16_bits_to_f32(got) - omr.bf16_bits_to_f32(exp))
    ulp = np.abs(omr.bf16_bits_to_f32(exp)) * 2.0 ** -7 + 1e-30
    assert np.all(diff <= ulp), float((diff / ulp).max())
    assert np.mean(got == exp) > 0.99
    # V rows moved verbatim, untouched rows unchanged
    assert np.array_equal(_bits(vd).reshape(NB * BS, -1)[dst.numpy()], _bits(vc).reshape(NB * BS, -1)[src.numpy()])
    others = np.setdiff1d(np.arange(NB * BS), dst.numpy())
    assert np.array_equal(_bits(kd).reshape(NB * BS, -1)[others], _bits(kc).reshape(NB * BS, -1)[others])


def test_mrope_shift_in_place_equals_rotation_at_new_position(ops):
    """Rotating K stored at offset 0 by delta 16 ~= rotating the raw K at offset 16 (cfg1)."""
    g = torch.Generator().manual_seed(0)
    raw = torch.randn(1024, 2, 128, generator=g)
    pos_old = omr.vision_positions(0, 32, 32)
    pos_new = omr.vision_positions(16, 32, 32)
    k_old = omr.apply_mrope(raw, pos_old).to(torch.bfloat16)
    k_new_ref = omr.apply_mrope(raw, pos_new)
    kc = torch.zeros(8, 256, 2, 128, dtype=torch.bfloat16)
    kc.view(-1, 2, 128)[:1024] = k_old
    kd = kc.cuda()
    ops.mrope_shift(kd, None, torch.arange(1024, dtype=torch.int32, device="cuda"), None, (16, 16, 16))
    got = kd.view(-1, 2, 128)[:1024].float().cpu()
    err = (got - k_new_ref).abs()
    x = k_old.float()
    bound = 2.0 ** -8 * (x.abs() + x.roll(64, dims=-1).abs() + k_new_ref.abs()) + 1e-6
    assert torch.all(err <= bound)


# ------------------------------------------------------------------ prefill attention
def _run_prefill(ops, case, H, Hk):
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda")
    out = ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return out, plan


@pytest.mark.parametrize("model", ["3b", "7b"])
def test_prefill_small_warm_requests(ops, model):
    cfg = QWEN_3B if model == "3b" else QWEN_7B
    H, Hk = cfg["num_heads"], cfg["num_kv_heads"]
    specs = [(16, 1024, 32, 102), (5, 300, 17, 30), (0, 200, 9, 1)]
    case = make_warm_case(specs, H, Hk, device="cuda", seed=3)
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    out, _ = _run_prefill(ops, case, H, Hk)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_nan_in_unwritten_slots(ops):
    """Slots past the sequence end hold NaN bit patterns; they must not leak into outputs."""
    H, Hk = 16, 2
    specs = [(16, 1024, 32, 102)]
    case = make_warm_case(specs, H, Hk, device="cpu", seed=4)
    n = 16 + 1024 + 32
    poison_unused_slots(case.k_cache, case.block_tables[1:2], [n])
    poison_unused_slots(case.v_cache, case.block_tables[1:2], [n])
    ref = oatt.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cu_q, case.cu_k,
                                 case.scale)
    case.q, case.k_cache, case.v_cache, case.block_tables = (case.q.cuda(), case.k_cache.cuda(),
                                                             case.v_cache.cuda(), case.block_tables.cuda())
    out, _ = _run_prefill(ops, case, H, Hk)
    assert torch.isfinite(out).all()
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_split_tiles_repeat_launches(ops):
    """Split tiles (partials merged by the merge kernel): repeated launches on the same
    workspace give identical results (as every layer of a step reuses it)."""
    H, Hk = 16, 2
    case = make_warm_case([(20, 4000, 48, 400)], H, Hk, device="cuda", seed=21)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda", num_sms=16)
    assert plan.num_merges > 0
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device="cuda")
    outs = [ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale,
                                  workspace=ws) for _ in range(3)]
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(outs[0], ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def _inflight_rows(case, H, Hk):
    """k_new / v_new as the projection would hold them: row i = key / value of query row i
    (gathered from the pages through the block table)."""
    bs = case.k_cache.shape[1]
    bt = case.block_tables.cpu().numpy()
    slots = []
    for b in range(len(case.cu_q) - 1):
        ql, kl = case.cu_q[b + 1] - case.cu_q[b], case.cu_k[b + 1] - case.cu_k[b]
        for t in range(ql):
            pos = kl - ql + t
            slots.append(int(bt[b][pos // bs]) * bs + pos % bs)
    idx = torch.tensor(slots, device=case.k_cache.device)
    D = case.k_cache.shape[-1]
    return case.k_cache.view(-1, Hk, D)[idx].contiguous(), case.v_cache.view(-1, Hk, D)[idx].contiguous()


def test_prefill_inflight_kv(ops):
    """vlc_prefill_attn_inflight: the first sub-sequence of each warm request (q_len ==
    k_len) reads its keys from the in-flight rows.  Its pages are replaced by NaN copies
    (a second block-table row), so the paged launch would fail there; the in-flight launch
    gives bit-for-bit the paged launch on the intact cache, split tiles included."""
    H, Hk = 16, 2
    case = make_warm_case([(16, 1024, 32, 102), (5, 2000, 17, 300), (0, 400, 9, 40)], H, Hk, device="cuda",
                          seed=31)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda", num_sms=32)
    assert plan.num_merges > 0
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device="cuda")
    ref = ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale,
                                workspace=ws)
    k_new, v_new = _inflight_rows(case, H, Hk)
    # NaN copies of every page the self-attention rows use, referenced only by their rows
    bt = case.block_tables.clone()
    nb = case.k_cache.shape[0]
    extra = []
    for b in range(len(case.cu_q) - 1):
        if case.cu_q[b + 1] - case.cu_q[b] != case.cu_k[b + 1] - case.cu_k[b]:
            continue
        for j in range(bt.shape[1]):
            if int(bt[b, j]) >= 0:
                extra.append(int(bt[b, j]))
                bt[b, j] = nb + len(extra) - 1
    assert extra
    nan_pages = torch.full((len(extra),) + tuple(case.k_cache.shape[1:]), float("nan"), dtype=torch.bfloat16,
                           device="cuda")
    kc = torch.cat([case.k_cache, nan_pages])
    vc = torch.cat([case.v_cache, nan_pages])
    out = ops.prefill_attention(case.q, kc, vc, bt, plan, case.scale, workspace=ws, k_new=k_new, v_new=v_new)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.isfinite(out.float()).all()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("num_sms", [148, 16])
def test_prefill_quad_units(ops, num_sms):
    """Quad units on CTA pairs (``PREFILL_QUADS``: clusters of 2, tcgen05.mma.cta_group::2,
    each CTA loading half of every K/V block, ghost tiles in short quads; with 16 SMs the
    long tiles split): against the oracle, and against the pairs kernel on the same inputs."""
    H, Hk = 16, 2
    case = make_warm_case([(16, 1024, 32, 102), (5, 300, 17, 30), (0, 200, 9, 1), (20, 4000, 48, 400)], H, Hk,
                          device="cuda", seed=23)
    outs = []
    for mode in (ops.PREFILL_PAIRS, ops.PREFILL_QUADS):
        ops.set_prefill_kernel(mode)
        try:
            plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda", num_sms=num_sms)
        finally:
            ops.set_prefill_kernel(ops.PREFILL_DEFAULT)
        assert int(plan.host[21]) == (1 if mode == ops.PREFILL_QUADS else 0)
        ws = torch.empty(max(1, plan.workspace_bytes), dtype=torch.uint8, device="cuda")
        outs.append(ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale,
                                          workspace=ws))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(outs[1], ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)
    assert float((outs[0].float() - outs[1].float()).abs().max()) <= ATT_MAX


def test_prefill_cfg2_full_size(ops):
    """BASELINE config 2 (3B, 4K image, 10% recompute): 1,123 query rows x 10,617 keys."""
    H, Hk = 16, 2
    case = make_warm_case(cfg2_spec(0.1), H, Hk, device="cuda", seed=5)
    out, plan = _run_prefill(ops, case, H, Hk)
    assert plan.num_merges > 0
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_full_causal_7b(ops):
    """Full (ratio 1.0) causal prefill over a 2.5k-token request, 7B heads."""
    H, Hk = 28, 4
    case = make_warm_case([(20, 2450, 48, 2450)], H, Hk, device="cuda", seed=6)
    out, _ = _run_prefill(ops, case, H, Hk)
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


@pytest.mark.parametrize("block_size", [128, 512])
def test_prefill_block_sizes_and_empty_sequences(ops, block_size):
    """Pages of 128 and 512 keys; empty virtual sequences (no suffix, no prefix) and keys
    ending on and off a 128-key boundary."""
    H, Hk = 16, 2
    specs = [(0, 640, 0, 64), (7, 121, 0, 121), (20, 500, 12, 0), (3, 250, 5, 40)]
    case = make_warm_case(specs, H, Hk, device="cuda", seed=8, block_size=block_size)
    assert any(case.cu_q[i + 1] == case.cu_q[i] for i in range(len(case.cu_q) - 1))
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    out, _ = _run_prefill(ops, case, H, Hk)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_long_keys_max_parts(ops):
    """48 text rows after a 40,000-token image: the long tiles split into the planner's
    maximum part count (one round of merge loads per lane group)."""
    H, Hk = 16, 2
    case = make_warm_case([(20, 40000, 48, 0)], H, Hk, device="cuda", seed=9)
    out, plan = _run_prefill(ops, case, H, Hk)
    h = plan.host
    merges = h[int(h[14]):int(h[14]) + plan.num_merges * 8].reshape(-1, 8)
    assert int(merges[:, 4].max()) == 20
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


@pytest.mark.parametrize("num_sms", [148, 16])
def test_prefill_split_back_to_back(ops, num_sms):
    """Launches with split tiles on one plan and workspace run back to back (each attention a
    programmatic dependent of the previous merge), eagerly and in a replayed graph, with
    different queries each time: every output equals that of a launch of its own."""
    H, Hk = 16, 2
    case = make_warm_case([(20, 6000, 48, 300), (0, 900, 64, 0)], H, Hk, device="cuda", seed=29)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda", num_sms=num_sms)
    assert plan.num_merges > 0
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device="cuda")
    qs = [case.q * s for s in (1.0, 0.5, -0.75, 1.25)]
    solo = []
    for q in qs:
        o = torch.empty_like(q)
        ops.prefill_attention(q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale, o, ws)
        torch.cuda.synchronize()
        solo.append(o)
    outs = [torch.empty_like(q) for q in qs]
    for q, o in zip(qs, outs):
        ops.prefill_attention(q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale, o, ws)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for o, r in zip(outs, solo):
        assert torch.equal(o, r)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for q, o in zip(qs, outs):
            ops.prefill_attention(q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale, o, ws)
    for _ in range(3):
        for o in outs:
            o.zero_()
        graph.replay()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for o, r in zip(outs, solo):
        assert torch.equal(o, r)
    ref = oatt.prefill_attention(qs[2].cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(outs[2], ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


# ------------------------------------------------------------------ decode
@pytest.mark.parametrize("model,lens", [("7b", [1, 63, 64, 65, 700, 2711, 5000, 10700]),
                                        ("3b", [255, 256, 257, 4097])])
def test_decode_matches_oracle(ops, model, lens):
    cfg = QWEN_3B if model == "3b" else QWEN_7B
    H, Hk = cfg["num_heads"], cfg["num_kv_heads"]
    q, kc, vc, bt, ctx, scale = make_decode_case(len(lens), H, Hk, lens, seed=7)
    poison_unused_slots(kc, bt, lens)
    poison_unused_slots(vc, bt, lens)
    ref = oatt.decode_attention(q, kc, vc, bt, ctx, scale)
    out = ops.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), bt.cuda(), ctx.cuda(), max(lens), scale)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert torch.isfinite(out).all()
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)


def test_prefill_graph_capture_replay(ops):
    """The prefill launch (attention + split merge) is capture-safe: a captured CUDA graph
    replays to the eager result, also after the inputs change in place (as the bench's
    per-step graph and nano-vllm's graphs use it)."""
    H, Hk = 16, 2
    case = make_warm_case([(20, 3000, 48, 300)], H, Hk, device="cuda", seed=23)
    plan = ops.build_prefill_plan(case.cu_q, case.cu_k, H, Hk, device="cuda", num_sms=32)
    assert plan.num_merges > 0
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(case.q)
    ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale, out, ws)
    torch.cuda.synchronize()
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, plan, case.scale, out, ws)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    case.q.mul_(0.5)
    graph.replay()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref = oatt.prefill_attention(case.q.cpu(), case.k_cache.cpu(), case.v_cache.cpu(), case.block_tables.cpu(),
                                 case.cu_q, case.cu_k, case.scale)
    mx, mean = attn_errors(out, ref)
    assert mx <= ATT_MAX and mean <= ATT_MEAN, (mx, mean)
