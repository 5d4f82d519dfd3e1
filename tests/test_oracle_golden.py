"""Pin the CPU oracle against the golden fixtures made from the reference's own code
(nano-vllm warm-prefill metadata) and from HF transformers' Qwen2.5-VL M-RoPE."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import metadata as omd
from oracle import mrope as omr
from oracle import rope as orope

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return dict(np.load(GOLD / name))


def _specs(g):
    specs = []
    for i, (n, s, e, R, partial) in enumerate(g["requests"]):
        bt = [int(x) for x in g["request_block_tables"][i] if x >= 0]
        specs.append(omd.SeqSpec(int(n), bt, int(s) if s >= 0 else None, int(e) if e >= 0 else None, int(R),
                                 bool(partial)))
    return specs


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "mixed"])
def test_prepare_prefill_matches_reference(name):
    g = _load(f"metadata_{name}.npz")
    meta = omd.prepare_prefill(_specs(g), int(g["block_size"]))
    assert np.array_equal(meta.cu_seqlens_q, g["cu_seqlens_q"])
    assert np.array_equal(meta.cu_seqlens_k, g["cu_seqlens_k"])
    assert meta.max_seqlen_q == int(g["max_seqlen_q"]) and meta.max_seqlen_k == int(g["max_seqlen_k"])
    assert np.array_equal(meta.slot_mapping, g["slot_mapping"])
    assert np.array_equal(meta.positions, g["positions"])
    if g["block_tables"].size:
        assert np.array_equal(meta.block_tables, g["block_tables"])
    assert list(meta.logit_indices or []) == list(g["logit_indices"])


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "mixed"])
def test_recompute_count_and_image_copy_slots(name):
    g = _load(f"metadata_{name}.npz")
    ratio = float(g["ratio"])
    olds, news = [], []
    for i, (n, s, e, R, partial) in enumerate(g["requests"]):
        if not partial:
            continue
        assert omd.recompute_count(ratio, int(e - s)) == int(R)
        bt = [int(x) for x in g["request_block_tables"][i] if x >= 0]
        o, nw = omd.image_kv_copy_slots(int(s), int(e), int(R), bt, int(g["cold_img_start"]),
                                        g["cold_block_table"], int(g["block_size"]))
        olds.append(o)
        news.append(nw)
    assert np.array_equal(np.concatenate(olds), g["old_slots"])
    assert np.array_equal(np.concatenate(news), g["new_slots"])


def test_cfg_recompute_counts():
    # BASELINE: cfg2 R = 1,055 of 10,549; cfg3 135 of 2,691; cfg4 211/528/1,055/10,549.
    assert omd.recompute_count(0.1, 10549) == 1055
    assert omd.recompute_count(0.05, 2691) == 135
    assert [omd.recompute_count(r, 10549) for r in (0.02, 0.05, 0.1, 1.0)] == [211, 528, 1055, 10549]
    # cfg1 under the reference rule is 103 (BASELINE's synthetic cfg1 queries 102 rows).
    assert omd.recompute_count(0.1, 1024) == 103


def test_prepare_decode_matches_reference():
    g = _load("metadata_decode.npz")
    bts = [[int(x) for x in row if x >= 0] for row in g["request_block_tables"]]
    pos, slot, lens, bt = omd.prepare_decode(g["seqlens"], bts)
    assert np.array_equal(pos, g["positions"])
    assert np.array_equal(slot, g["slot_mapping"])
    assert np.array_equal(lens, g["context_lens"])
    assert np.array_equal(bt, g["block_tables"])


def test_mrope_matches_hf():
    g = _load("mrope_cfg1.npz")
    assert np.array_equal(omr.vision_positions(0, 32, 32), g["pos_old"])
    assert np.array_equal(omr.vision_positions(16, 32, 32), g["pos_new"])
    assert np.allclose(omr.inv_freq(128, 1e6).numpy(), g["inv_freq"], rtol=0, atol=0)
    raw = torch.randn(1, 2, 1024, 128, generator=torch.Generator().manual_seed(0))
    assert abs(float(raw.double().sum()) - float(g["raw_checksum"])) < 1e-6
    raw = raw[0].permute(1, 0, 2)
    k_old = omr.apply_mrope(raw, omr.vision_positions(0, 32, 32))[::8]
    k_new = omr.apply_mrope(raw, omr.vision_positions(16, 32, 32))[::8]
    assert torch.allclose(k_old, torch.from_numpy(g["k_old"]), atol=2e-6, rtol=0)
    assert torch.allclose(k_new, torch.from_numpy(g["k_new"]), atol=2e-6, rtol=0)


def test_shift_restatement_reaches_hf_new_position():
    """Rotating the bf16-stored K(old) by delta 16 lands on HF's K(new) within the bf16 bound."""
    g = _load("mrope_cfg1.npz")
    k_old = torch.from_numpy(g["k_old"])
    bits = omr.f32_to_bf16_bits(k_old.numpy())
    shifted = omr.bf16_bits_to_f32(omr.shift_rows(bits, (16, 16, 16)))
    ref = g["k_new"]
    x = omr.bf16_bits_to_f32(bits)
    bound = 2.0 ** -8 * (np.abs(x) + np.abs(np.roll(x, 64, axis=-1)) + np.abs(ref)) + 1e-6
    assert np.all(np.abs(shifted - ref) <= bound)


def test_shift_composition_identity():
    """R(a)R(b) = R(a+b): shifting by d1 then d2 equals shifting by d1+d2 (to bf16 rounding)."""
    rng = np.random.default_rng(0)
    bits = omr.f32_to_bf16_bits(rng.standard_normal((64, 2, 128)).astype(np.float32))
    a = omr.bf16_bits_to_f32(omr.shift_rows(omr.shift_rows(bits, (3, 5, 7)), (4, -2, 9)))
    b = omr.bf16_bits_to_f32(omr.shift_rows(bits, (7, 3, 16)))
    assert np.max(np.abs(a - b)) < 0.05
    z = omr.shift_rows(bits, (0, 0, 0))
    assert np.array_equal(z, bits)


def test_attention_oracle_regression_cfg1():
    from tests.helpers import make_cfg1_case
    g = _load("attention_cfg1.npz")
    case = make_cfg1_case(dtype=torch.float32)
    assert np.array_equal(case.cu_q, g["cu_q"]) and np.array_equal(case.cu_k, g["cu_k"])
    out = oatt.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cu_q, case.cu_k,
                                 case.scale)
    assert np.allclose(out.sum(-1).numpy(), g["row_sum"], atol=1e-4)
    assert np.allclose((out * out).sum(-1).numpy(), g["row_sq"], atol=1e-4)
    assert np.allclose(out[::19].numpy(), g["rows"], atol=1e-5)


def test_attention_oracle_semantics_small():
    """Bottom-right causal: a query row with logical position p equals full softmax over keys [0, p]."""
    g = torch.Generator().manual_seed(3)
    k = torch.randn(1, 256, 1, 128, generator=g)
    v = torch.randn(1, 256, 1, 128, generator=g)
    q = torch.randn(3, 2, 128, generator=g)
    cu_q, cu_k = [0, 3], [0, 200]
    out = oatt.prefill_attention(q, k, v, [[0]], cu_q, cu_k, 0.1)
    for i, p in enumerate(range(197, 200)):
        s = (q[i] @ k[0, :p + 1, 0].T) * 0.1
        ref = torch.softmax(s, -1) @ v[0, :p + 1, 0]
        assert torch.allclose(out[i], ref, atol=1e-5)
    assert oatt.causal_pairs([0, 1075, 1123], [0, 1075, 11692]) == 1086838


def test_rope_oracle_and_table_match_reference():
    """nano-vllm's RoPE (rotary_embedding.py:6-14, 29-48), evaluated eagerly by the
    reference itself: the cos/sin table this package builds and the oracle's rotation
    match it bit for bit."""
    from vlcache_b200.layers.rotary_embedding import rope_cos_sin_cache
    f = np.load(GOLD / "rope_3b.npz")
    table = rope_cos_sin_cache(128, int(f["max_position"]), 1e6)
    pos = f["positions"]
    assert table.shape == (int(f["max_position"]), 1, 128) and table.dtype == torch.float32
    assert np.array_equal(table[pos, 0].numpy().view(np.uint32), f["cos_sin_rows"].view(np.uint32))
    assert np.array_equal(orope.rope_rows(f["q"], pos, table[:, 0].numpy()), f["q_rot"])
    assert np.array_equal(orope.rope_rows(f["k"], pos, table[:, 0].numpy()), f["k_rot"])


def test_rope_store_oracle_skips_minus_one_slots():
    g = np.random.default_rng(3)
    n, hk, d = 5, 2, 128
    table = np.zeros((16, d), np.float32)
    table[:, : d // 2] = 1.0                       # cos 1, sin 0: rotation is the identity
    q = g.integers(0, 0x4000, (n, 4, d), dtype=np.uint16)
    k = g.integers(0, 0x4000, (n, hk, d), dtype=np.uint16)
    v = g.integers(0, 0x4000, (n, hk, d), dtype=np.uint16)
    kc = np.zeros((8, hk * d), np.uint16)
    q_out, kc2, vc2 = orope.rope_store_kvcache(np.arange(n), q, k, v, table, kc, kc, np.array([3, -1, 0, 7, -1]))
    assert np.array_equal(q_out, q)
    assert np.array_equal(kc2[[3, 0, 7]], k[[0, 2, 3]].reshape(3, -1))
    assert np.array_equal(vc2[[3, 0, 7]], v[[0, 2, 3]].reshape(3, -1))
    assert not kc2[[1, 2, 4, 5, 6]].any()
