"""Host logic of the product (no GPU): metadata builder, image-reuse slots, the
attention planner (through the C ABI), and the loud failure of the CUDA-only ops."""
from pathlib import Path

import numpy as np
import pytest
import torch

from vlcache_b200.engine import kv_cache as kvc

GOLD = Path(__file__).resolve().parent / "golden"


def _reqs(g):
    out = []
    for i, (n, s, e, R, partial) in enumerate(g["requests"]):
        bt = [int(x) for x in g["request_block_tables"][i] if x >= 0]
        out.append(kvc.WarmRequest(int(n), bt, int(s) if s >= 0 else None, int(e) if e >= 0 else None, int(R),
                                   bool(partial)))
    return out


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "mixed"])
def test_builder_bit_exact_vs_reference(name):
    g = dict(np.load(GOLD / f"metadata_{name}.npz"))
    b = kvc.WarmPrefillBuilder(16, 2).build(_reqs(g))
    assert np.array_equal(b.cu_seqlens_q, g["cu_seqlens_q"])
    assert np.array_equal(b.cu_seqlens_k, g["cu_seqlens_k"])
    assert np.array_equal(b.slot_mapping, g["slot_mapping"])
    assert np.array_equal(b.positions, g["positions"])
    assert np.array_equal(b.block_tables, g["block_tables"])
    assert b.max_seqlen_q == int(g["max_seqlen_q"]) and b.max_seqlen_k == int(g["max_seqlen_k"])
    assert list(b.logit_indices) == list(g["logit_indices"])


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "mixed"])
def test_image_reuse_slots_vs_reference(name):
    g = dict(np.load(GOLD / f"metadata_{name}.npz"))
    src, dst = [], []
    for r in _reqs(g):
        if r.partial:
            s, d = kvc.image_reuse_slots(r.img_start, r.img_end, r.num_recompute, r.block_table,
                                         int(g["cold_img_start"]), g["cold_block_table"])
            src.append(s)
            dst.append(d)
    assert np.array_equal(np.concatenate(src), g["old_slots"])
    assert np.array_equal(np.concatenate(dst), g["new_slots"])
    # new pages are freshly allocated: source and destination never overlap
    assert not set(np.concatenate(src).tolist()) & set(np.concatenate(dst).tolist())


def test_recompute_count():
    assert kvc.recompute_count(0.1, 10549) == 1055
    assert kvc.recompute_count(0.05, 2691) == 135


# ---------------------------------------------------------------- planner (C ABI, host only)
UNIT_INTS, MERGE_INTS = 17, 8


def _decode_plan(plan):
    from vlcache_b200 import ops  # noqa: F401  (loads the library)
    h = plan.host
    grid, nu, nparts, nm = int(h[2]), int(h[3]), int(h[4]), int(h[5])
    cta = h[int(h[12]):int(h[12]) + grid + 1]
    units = h[int(h[13]):int(h[13]) + nu * UNIT_INTS].reshape(nu, UNIT_INTS)
    merges = h[int(h[14]):int(h[14]) + nm * MERGE_INTS].reshape(nm, MERGE_INTS)
    return grid, cta, units, merges, nparts


def _unit_tiles(u):
    """(q_begin, q_count, kpos0, part, kb_begin, kb_end) of the tiles of a unit."""
    seq, g, kb0, kb1, kvl, kbase, cost = [int(x) for x in u[:7]]
    out = [(int(u[7]), int(u[8]), int(u[9]), int(u[10]), kb0, kb1)]
    if int(u[12]) > 0:
        out.append((int(u[11]), int(u[12]), int(u[13]), int(u[14]), kb0, int(u[15])))
    return out


def _coverage(cu_q, cu_k, H, Hk, num_sms, causal=True, head_dim=128):
    from vlcache_b200 import ops
    plan = ops.build_prefill_plan(cu_q, cu_k, H, Hk, head_dim, num_sms=num_sms, causal=causal)
    assert int(plan.host[18]) == int(causal) and int(plan.host[19]) == head_dim
    grid, cta, units, merges, nparts = _decode_plan(plan)
    G = H // Hk
    T = 128 // G
    assert int(plan.host[6]) == T * G and int(plan.host[7]) == T
    assert cta[0] == 0 and cta[-1] == len(units) and np.all(np.diff(cta) >= 0)
    assert grid <= num_sms
    # every (query token, kv head, key block) visible under the causal mask is covered exactly once
    need = {}
    for b in range(len(cu_q) - 1):
        ql, kl = cu_q[b + 1] - cu_q[b], cu_k[b + 1] - cu_k[b]
        for g in range(Hk):
            for t in range(ql):
                pos = kl - ql + t if causal else kl - 1
                for kb in range(pos // 128 + 1):
                    need[(cu_q[b] + t, g, kb)] = 0
    parts_seen = set()
    # self-attention sequences (q_len == k_len) name their first row (in-flight K/V)
    for u in units:
        seq, g = int(u[0]), int(u[1])
        assert int(u[4]) == cu_k[seq + 1] - cu_k[seq] and int(u[5]) == cu_k[seq]
        ql, kl = cu_q[seq + 1] - cu_q[seq], cu_k[seq + 1] - cu_k[seq]
        assert int(u[16]) == (cu_q[seq] if ql == kl else -1)
        tiles = _unit_tiles(u)
        assert tiles[0][5] > tiles[0][4]                    # tile A always has work
        if len(tiles) == 2:
            assert tiles[1][0] + tiles[1][1] <= tiles[0][0]  # B holds the earlier tokens
            assert tiles[1][5] <= tiles[0][5]
        for (qb, qc, kp0, part, kb0, kb1) in tiles:
            assert 1 <= qc <= T
            for t in range(qc):
                for kb in range(kb0, kb1):
                    key = (qb + t, g, kb)
                    if key in need:
                        need[key] += 1
            if part >= 0:
                assert part not in parts_seen
                parts_seen.add(part)
    assert all(v == 1 for v in need.values())
    assert parts_seen == set(range(nparts))
    for m in merges:
        assert m[4] >= 2
        assert m[5] in (1, 2, 4) and m[6] == m[1] * G
    # merge launch: (merge << 8 | first row) per 8-warp block covers every valid row once
    h = plan.host
    nblk, off = int(h[16]), int(h[17])
    seen = {}
    for e in h[off:off + nblk]:
        mi, r0 = int(e) >> 8, int(e) & 255
        rpb = 8 * int(merges[mi][5])
        for r in range(r0, min(r0 + rpb, int(merges[mi][6]))):
            seen[(mi, r)] = seen.get((mi, r), 0) + 1
    assert seen == {(mi, r): 1 for mi in range(len(merges)) for r in range(int(merges[mi][6]))}
    return plan


@pytest.mark.parametrize("H,Hk", [(16, 2), (28, 4)])
def test_planner_covers_causal_pairs_exactly_once(H, Hk):
    cu_q = [0, 118, 150, 150 + 300, 150 + 300 + 9]
    cu_k = [0, 118, 118 + 1072, 118 + 1072 + 300, 118 + 1072 + 300 + 509]
    _coverage(cu_q, cu_k, H, Hk, num_sms=16)


@pytest.mark.parametrize("H,Hk,d", [(16, 16, 80), (16, 2, 128), (28, 4, 96)])
def test_planner_covers_noncausal_pairs_exactly_once(H, Hk, d):
    """Non-causal plans (vision windows and full attention): every key block of a
    sequence, for every query row of it, exactly once; ragged windows included."""
    lens = [64, 64, 37, 64, 300, 1, 64, 129]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    plan = _coverage(cu, cu, H, Hk, num_sms=16, causal=False, head_dim=d)
    units = _decode_plan(plan)[2]
    for u in units:
        for (_, _, kp0, _, _, _) in _unit_tiles(u):
            assert kp0 == int(u[4]) - 1          # non-causal rows see the whole sequence


def test_planner_head_dims():
    from vlcache_b200 import ops
    from vlcache_b200._lib import VLCError
    for d in (80, 96, 112, 128):
        ops.build_prefill_plan([0, 64], [0, 64], 16, 16, d, causal=False)
    for d in (64, 72, 136):
        with pytest.raises((ValueError, VLCError)):
            ops.build_prefill_plan([0, 64], [0, 64], 16, 16, d, causal=False)


def test_planner_cfg2_balanced():
    cu_q, cu_k = [0, 1075, 1123], [0, 1075, 11692]
    plan = _coverage(cu_q, cu_k, 16, 2, num_sms=148)
    grid, cta, units, merges, _ = _decode_plan(plan)
    loads = [units[cta[i]:cta[i + 1], 6].sum() / 16.0 for i in range(grid)]
    assert grid == 148 and max(loads) <= 1.6 * np.mean(loads)
    assert plan.workspace_bytes == plan.num_parts * 128 * (128 * 2 + 8)


def test_planner_rejects_bad_metadata():
    from vlcache_b200 import ops
    from vlcache_b200._lib import VLCError
    with pytest.raises((ValueError, VLCError)):
        ops.build_prefill_plan([0, 10], [0, 5], 16, 2)      # more queries than keys
    with pytest.raises((ValueError, VLCError)):
        ops.build_prefill_plan([1, 10], [0, 20], 16, 2)     # cu_seqlens must start at 0
    with pytest.raises((ValueError, VLCError)):
        ops.build_prefill_plan([0, 10], [0, 20], 16, 3)     # heads not divisible


def test_planner_empty_and_zero_length():
    from vlcache_b200 import ops
    plan = ops.build_prefill_plan([0, 0, 5], [0, 7, 12], 16, 2, num_sms=8)
    grid, cta, units, merges, _ = _decode_plan(plan)
    assert len(units) == 2 and all(int(u[0]) == 1 for u in units)   # one single-tile unit per KV head
    plan = ops.build_prefill_plan([0], [0], 16, 2, num_sms=8)
    assert plan.grid == 0


def test_ops_reject_cpu_tensors():
    """The product has no CPU path: CPU tensors fail loudly instead of silently falling back."""
    from vlcache_b200 import ops
    k = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    kc = torch.zeros(2, 256, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.store_kvcache(k, k, kc, kc, torch.zeros(4, dtype=torch.int32))
    from vlcache_b200.layers.rotary_embedding import RotaryEmbedding
    rot = RotaryEmbedding(128, 128, 64, 1e6)
    pos = torch.zeros(4, dtype=torch.int64)
    q = torch.zeros(4, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        rot(pos, q, k)
    with pytest.raises(ValueError):
        ops.rope_store_kvcache(pos, q, k, k, rot.cos_sin_cache, kc, kc, torch.zeros(4, dtype=torch.int32))


def test_reuse_slot_overlap_check():
    """Old and new block tables that share a page: rows moved onto themselves pass; a
    destination that is another row's source (image at a different offset in the shared
    page) is rejected before any launch."""
    from vlcache_b200.engine import kv_cache as kvc
    bt_old = [7, 3, 9]
    # same image position, page 3 shared: rows in page 3 move onto themselves
    src, dst = kvc.image_reuse_slots(20, 700, 5, [11, 3, 12], 20, bt_old)
    kvc.check_reuse_slots(src, dst)
    # image moved by 8 positions inside the shared page 3: slot overlap across rows
    src, dst = kvc.image_reuse_slots(28, 708, 5, [11, 3, 12], 20, bt_old)
    with pytest.raises(ValueError, match="overlap"):
        kvc.check_reuse_slots(src, dst)
    # disjoint pages: fine
    src, dst = kvc.image_reuse_slots(28, 708, 5, [11, 13, 12], 20, bt_old)
    kvc.check_reuse_slots(src, dst)
    with pytest.raises(ValueError, match="overlap"):
        kvc.copy_image_kv(torch.empty(2, 1, 16, 256, 2, 128), *kvc.image_reuse_slots(28, 708, 5, [11, 3, 12], 20,
                                                                                        bt_old))


def test_cache_budget_matches_reference_rule():
    """The sizing rule of nanovllm/engine/model_runner.py:130-151 on fixed memory figures
    (3B shapes: 36 layers, Hk 2, D 128, hidden 2048; a 180 GiB device)."""
    from vlcache_b200.engine import kv_cache as kvc
    GiB = 2 ** 30
    total, free = 180 * GiB, 172 * GiB
    peak, current = 9 * GiB, 7 * GiB
    b = kvc.cache_budget(36, 2, 128, 2048, mem_info=(free, total), peak_bytes=peak, current_bytes=current,
                         gpu_memory_utilization=0.9, encoder_cache_ratio=0.2)
    available = total * 0.9 - (total - free) - peak + current
    kv_block = 2 * 36 * 256 * 2 * 128 * 2
    enc_block = 256 * 2048 * 2
    assert b.kv_block_bytes == kv_block and b.encoder_block_bytes == enc_block
    assert b.num_kvcache_blocks == int(available - available * 0.2) // kv_block
    assert b.num_encoder_blocks == int(available * 0.2) // enc_block
    with pytest.raises(ValueError):
        kvc.cache_budget(36, 2, 128, 2048, mem_info=(1 * GiB, 180 * GiB), peak_bytes=0, current_bytes=0)


@pytest.mark.parametrize("H,Hk,lens", [(16, 16, [64, 64, 37, 64, 16, 1, 64, 48, 128]),
                                        (16, 2, [16, 3, 16, 9, 7, 16, 1])])
def test_planner_packs_short_noncausal_sequences(H, Hk, lens):
    """Non-causal self-attention of sequences that fit a tile (vision windows) packs whole
    consecutive sequences into single-block tiles, two independent tiles of one KV head per
    unit (each with the key block of its own rows); every token is in exactly one tile per
    KV head, and the plan's segment table gives each token its sequence's bounds."""
    from vlcache_b200 import ops
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    plan = ops.build_prefill_plan(cu, cu, H, Hk, 128, num_sms=8, causal=False)
    grid, cta, units, merges, nparts = _decode_plan(plan)
    T = 128 // (H // Hk)
    assert nparts == 0 and len(merges) == 0
    seen = np.zeros((int(cu[-1]), Hk), np.int32)
    starts = set(cu[:-1].tolist())
    for u in units:
        assert int(u[0]) == -1 and int(u[3]) - int(u[2]) == 1                      # packed, one block
        q0, qc = int(u[7]), int(u[8])
        assert 0 < qc <= T and q0 in starts and (q0 + qc) in set(cu.tolist())   # whole sequences
        assert int(u[4]) == qc and int(u[5]) == q0                               # tile A's keys: its rows
        seen[q0:q0 + qc, int(u[1])] += 1
        if int(u[12]) > 0:                                                       # tile B: its own rows
            qb, qcb = int(u[11]), int(u[12])
            assert 0 < qcb <= T and qb in starts and (qb + qcb) in set(cu.tolist()) and int(u[15]) == 1
            seen[qb:qb + qcb, int(u[1])] += 1
    assert np.all(seen == 1)
    off = int(plan.host[20])
    seg = plan.host[off:off + 2 * int(cu[-1])].reshape(-1, 2)
    for b in range(len(lens)):
        assert np.all(seg[cu[b]:cu[b + 1]] == [cu[b], cu[b + 1]])
    # a causal plan, or one with a sequence longer than a tile, is not packed
    assert int(ops.build_prefill_plan(cu, cu, H, Hk, 128, num_sms=8, causal=True).host[20]) == 0
    longer = np.array([0, T + 1], np.int32)
    assert int(ops.build_prefill_plan(longer, longer, H, Hk, 128, num_sms=8, causal=False).host[20]) == 0


@pytest.mark.parametrize("H,Hk", [(16, 2), (28, 4)])
def test_planner_quads_cover_pairs_exactly_once(H, Hk):
    """Quad plans (CTA pairs): unit i is records 2i (even CTA) and 2i + 1 (odd CTA), sharing
    sequence, KV head and key ranges; real tiles cover every visible (query token, KV head,
    key block) exactly once, ghost tiles (part -2) only stand in on the odd CTA; CTA ranges
    index CTA pairs and the grid is even."""
    from vlcache_b200 import ops
    cu_q = [0, 118, 150, 150 + 300, 150 + 300 + 9, 150 + 300 + 9 + 33]
    cu_k = [0, 118, 118 + 1072, 118 + 1072 + 300, 118 + 1072 + 300 + 509, 118 + 1072 + 300 + 509 + 4000]
    ops.set_prefill_kernel(ops.PREFILL_QUADS)
    try:
        plan = ops.build_prefill_plan(cu_q, cu_k, H, Hk, num_sms=32)
    finally:
        ops.set_prefill_kernel(ops.PREFILL_DEFAULT)
    h = plan.host
    assert int(h[21]) == 1
    grid, nrec = int(h[2]), int(h[3])
    assert grid % 2 == 0 and nrec % 2 == 0 and grid <= 32
    cta = h[int(h[12]):int(h[12]) + grid // 2 + 1]
    assert cta[0] == 0 and cta[-1] == nrec // 2 and np.all(np.diff(cta) >= 0)
    recs = h[int(h[13]):int(h[13]) + nrec * UNIT_INTS].reshape(nrec, UNIT_INTS)
    G, T = H // Hk, 128 // (H // Hk)
    need = {}
    for b in range(len(cu_q) - 1):
        ql, kl = cu_q[b + 1] - cu_q[b], cu_k[b + 1] - cu_k[b]
        for g in range(Hk):
            for t in range(ql):
                for kb in range((kl - ql + t) // 128 + 1):
                    need[(cu_q[b] + t, g, kb)] = 0
    for i in range(nrec // 2):
        ev, od = recs[2 * i], recs[2 * i + 1]
        for f in (0, 1, 2, 3, 4, 5, 15):               # seq, head, key range, kv_len, base, B's end
            assert ev[f] == od[f]
        assert (ev[12] > 0) == (od[12] > 0)             # both CTAs have a tile B, or neither
        assert ev[10] != -2 and ev[14] != -2            # ghosts only on the odd CTA
        for r in (ev, od):
            tiles = _unit_tiles(r)
            for ti, (qb, qc, kp0, part, kb0, kb1) in enumerate(tiles):
                if part == -2:
                    continue
                assert 1 <= qc <= T
                for t in range(qc):
                    for kb in range(kb0, kb1):
                        key = (qb + t, int(r[1]), kb)
                        if key in need:
                            need[key] += 1
    assert all(v == 1 for v in need.values())
