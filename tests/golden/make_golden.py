"""Generate the golden fixtures of tests/golden from the REFERENCE's own code.

Run here (where the reference tree and HF transformers are importable):
    python tests/golden/make_golden.py --reference <path to the VLCache checkout>

What is captured (all small):
  * metadata_*.npz — outputs of nano-vllm's pure-Python warm-prefill path run for
    synthetic requests: BlockManager.try_partial_recompute / allocate / store_image_kv
    (nanovllm/engine/block_manager.py), Sequence.find_image_token_range
    (nanovllm/engine/sequence.py:91-100), ModelRunner.prepare_prefill
    (nanovllm/engine/model_runner.py:194-320; its device copies are redirected to
    host tensors), LLMEngine._do_image_kv_copy (nanovllm/engine/llm_engine.py:58-89)
    and ModelRunner.prepare_decode (model_runner.py:322-338).
  * mrope_cfg1.npz — HF transformers' Qwen2.5-VL multimodal RoPE
    (Qwen2_5_VLRotaryEmbedding + apply_multimodal_rotary_pos_emb +
    get_vision_position_ids) applied to seeded keys of a 32x32 merged grid at vision
    start 0 and at start 16.
  * rope_3b.npz — nano-vllm's own 1-D RoPE (nanovllm/layers/rotary_embedding.py):
    rows of the ``RotaryEmbedding`` cos_sin_cache buffer (:29-35, theta 1e6, head 128)
    at seeded positions, and ``apply_rotary_emb`` (:6-14) of seeded bf16 query/key rows
    with cos | sin gathered as ``forward`` does (:37-48), evaluated eagerly on the CPU.
  * attention_cfg1.npz — checksums of the fp32 oracle attention of config 1
    (the reference's flash-attn path needs a GPU; the attention oracle is a
    restatement, so this file is a regression pin for it).
The fixtures are committed; tests never import the reference.
"""
from __future__ import annotations

import argparse
import contextlib
import math
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
IMAGE_TOKEN = 151655


@contextlib.contextmanager
def host_only_torch():
    """Let prepare_prefill/prepare_decode run without a GPU: drop pin_memory and make
    .cuda() a no-op for the duration."""
    orig_tensor = torch.tensor
    orig_cuda = torch.Tensor.cuda

    def tensor(*a, **kw):
        kw.pop("pin_memory", None)
        return orig_tensor(*a, **kw)

    torch.tensor = tensor
    torch.Tensor.cuda = lambda self, *a, **kw: self
    try:
        yield
    finally:
        torch.tensor = orig_tensor
        torch.Tensor.cuda = orig_cuda


def make_tokens(prefix, n_img, suffix, base=1000):
    return list(range(base, base + prefix)) + [IMAGE_TOKEN] * n_img + list(range(base + 50000, base + 50000 + suffix))


def run_metadata_scenario(name, cold_prefix, warm_specs, ratio, num_blocks=400, block_size=256, seed=0):
    """One cold request caches the image; warm requests reuse it (possibly at other offsets)."""
    from nanovllm.engine.block_manager import BlockManager
    from nanovllm.engine.llm_engine import LLMEngine
    from nanovllm.engine.model_runner import ModelRunner
    from nanovllm.engine.sequence import Sequence
    from nanovllm.utils.context import get_context

    rng = np.random.default_rng(seed)
    bm = BlockManager(num_blocks, block_size, ratio)
    # Shuffle the free list so block tables are not the identity.
    perm = rng.permutation(num_blocks).tolist()
    bm.free_block_ids.clear()
    bm.free_block_ids.extend(perm)
    img_hash = 0x1234ABCD
    n_img = warm_specs[0][1]
    cold = Sequence(make_tokens(cold_prefix, n_img, 7), image_hashes=[img_hash])
    bm.allocate(cold)
    cold.find_image_token_range(IMAGE_TOKEN)
    bm.store_image_kv(cold)

    seqs = []
    for (prefix, ni, suffix, has_image) in warm_specs:
        if has_image:
            s = Sequence(make_tokens(prefix, ni, suffix), image_hashes=[img_hash])
            hit = bm.try_partial_recompute(s, IMAGE_TOKEN)
            assert hit
        else:
            s = Sequence(list(range(5, 5 + prefix + suffix)))
        bm.allocate(s)
        seqs.append(s)

    runner = object.__new__(ModelRunner)
    runner.block_size = block_size
    with host_only_torch():
        input_ids, positions, _ = runner.prepare_prefill(seqs)
        ctx = get_context()
        copies = []
        eng = object.__new__(LLMEngine)
        eng.scheduler = SimpleNamespace(block_manager=bm)
        eng.model_runner = SimpleNamespace(call=lambda fn, *a: copies.append(a))
        eng._do_image_kv_copy(seqs)
    old_slots = np.concatenate([np.asarray(c[0], np.int32) for c in copies]) if copies else np.zeros(0, np.int32)
    new_slots = np.concatenate([np.asarray(c[1], np.int32) for c in copies]) if copies else np.zeros(0, np.int32)

    req = []
    for s in seqs:
        rng_ = s.image_token_range if s.image_token_range is not None else (-1, -1)
        req.append([len(s), rng_[0], rng_[1], s.num_recompute_tokens, int(s.is_partial_recompute)])
    width = max(len(s.block_table) for s in seqs)
    bts = np.full((len(seqs), width), -1, np.int32)
    for i, s in enumerate(seqs):
        bts[i, :len(s.block_table)] = s.block_table
    out = dict(
        requests=np.asarray(req, np.int64),
        request_block_tables=bts,
        cold_img_start=np.int64(cold.image_token_range[0]),
        cold_block_table=np.asarray(cold.block_table, np.int32),
        positions=positions.numpy().astype(np.int64),
        cu_seqlens_q=ctx.cu_seqlens_q.numpy().astype(np.int32),
        cu_seqlens_k=ctx.cu_seqlens_k.numpy().astype(np.int32),
        max_seqlen_q=np.int64(ctx.max_seqlen_q),
        max_seqlen_k=np.int64(ctx.max_seqlen_k),
        slot_mapping=ctx.slot_mapping.numpy().astype(np.int32),
        block_tables=(ctx.block_tables.numpy().astype(np.int32) if ctx.block_tables is not None
                      else np.zeros((0, 0), np.int32)),
        logit_indices=np.asarray(runner._logit_indices or [], np.int64),
        old_slots=old_slots,
        new_slots=new_slots,
        ratio=np.float64(ratio),
        block_size=np.int64(block_size),
    )
    np.savez_compressed(HERE / f"metadata_{name}.npz", **out)
    return out


def run_decode_scenario(block_size=256):
    from nanovllm.engine.block_manager import BlockManager
    from nanovllm.engine.model_runner import ModelRunner
    from nanovllm.engine.sequence import Sequence
    from nanovllm.utils.context import get_context

    bm = BlockManager(64, block_size, 0.0)
    lens = [1, 255, 256, 257, 700, 513]
    seqs = []
    for n in lens:
        s = Sequence(list(range(3, 3 + n)))
        bm.allocate(s)
        s.append_token(7)      # one generated token: decode writes its K/V
        bm.may_append(s)
        seqs.append(s)
    runner = object.__new__(ModelRunner)
    runner.block_size = block_size
    with host_only_torch():
        input_ids, positions = runner.prepare_decode(seqs)
        ctx = get_context()
    width = max(len(s.block_table) for s in seqs)
    bts = np.full((len(seqs), width), -1, np.int32)
    for i, s in enumerate(seqs):
        bts[i, :len(s.block_table)] = s.block_table
    np.savez_compressed(HERE / "metadata_decode.npz",
                        seqlens=np.asarray([len(s) for s in seqs], np.int64),
                        request_block_tables=bts,
                        positions=positions.numpy().astype(np.int64),
                        slot_mapping=ctx.slot_mapping.numpy().astype(np.int32),
                        context_lens=ctx.context_lens.numpy().astype(np.int32),
                        block_tables=ctx.block_tables.numpy().astype(np.int32))


def run_mrope_cfg1():
    from transformers.models.qwen2_5_vl import modeling_qwen2_5_vl as hf
    from transformers.models.qwen2_5_vl.configuration_qwen2_5_vl import Qwen2_5_VLTextConfig

    cfg = Qwen2_5_VLTextConfig(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2,
                               rope_parameters={"rope_type": "default", "rope_theta": 1e6,
                                                "mrope_section": [16, 24, 24]})
    rot = hf.Qwen2_5_VLRotaryEmbedding(cfg)
    grid = torch.tensor([1, 64, 64])       # 64x64 patches, 2x2 merge -> 32x32 tokens
    pos_old = hf.Qwen2_5_VLModel.get_vision_position_ids(None, 0, grid, 1, 2)
    pos_new = hf.Qwen2_5_VLModel.get_vision_position_ids(None, 16, grid, 1, 2)
    g = torch.Generator().manual_seed(0)
    raw = torch.randn(1, 2, 1024, 128, generator=g)        # [batch, kv heads, tokens, dim]
    q_dummy = torch.zeros(1, 1, 1024, 128)
    outs = {}
    for tag, pos in (("old", pos_old), ("new", pos_new)):
        cos, sin = rot(raw, pos[:, None, :])
        _, k_rot = hf.apply_multimodal_rotary_pos_emb(q_dummy, raw, cos, sin, [16, 24, 24])
        outs[tag] = k_rot[0].permute(1, 0, 2).contiguous()  # [tokens, heads, dim]
    # raw keys are regenerated from the seed by the tests (torch.randn, seed 0, shape
    # [1, 2, 1024, 128]); every 8th token is stored to keep the fixture small.
    sel = slice(None, None, 8)
    np.savez_compressed(HERE / "mrope_cfg1.npz",
                        raw_checksum=np.float64(raw.double().sum()),
                        pos_old=pos_old.numpy().astype(np.int32), pos_new=pos_new.numpy().astype(np.int32),
                        k_old=outs["old"][sel].numpy().astype(np.float32),
                        k_new=outs["new"][sel].numpy().astype(np.float32),
                        inv_freq=rot.inv_freq.numpy().astype(np.float32))


def run_rope():
    from nanovllm.layers.rotary_embedding import RotaryEmbedding, apply_rotary_emb

    max_pos = 32768
    rot = RotaryEmbedding(128, 128, max_pos, 1e6)   # only the table: forward is torch.compile'd
    g = torch.Generator().manual_seed(7)
    n, h, hk = 24, 4, 2
    pos = torch.randint(0, max_pos, (n,), generator=g, dtype=torch.int64)
    pos[:4] = torch.tensor([0, 1, max_pos - 1, 10617])
    q = torch.randn(n, h, 128, generator=g).mul_(3).to(torch.bfloat16)
    k = torch.randn(n, hk, 128, generator=g).mul_(3).to(torch.bfloat16)
    cos, sin = rot.cos_sin_cache[pos].chunk(2, dim=-1)       # as forward (:44-45)
    q_ref = apply_rotary_emb(q, cos, sin)
    k_ref = apply_rotary_emb(k, cos, sin)
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(HERE / "rope_3b.npz", max_position=np.int64(max_pos), positions=pos.numpy(),
                        cos_sin_rows=rot.cos_sin_cache[pos, 0].numpy().astype(np.float32),
                        q=bits(q), k=bits(k), q_rot=bits(q_ref), k_rot=bits(k_ref))


def run_attention_cfg1():
    sys.path.insert(0, str(REPO))
    from oracle import attention as oatt
    from tests.helpers import make_cfg1_case
    case = make_cfg1_case(dtype=torch.float32)
    out = oatt.prefill_attention(case.q, case.k_cache, case.v_cache, case.block_tables, case.cu_q, case.cu_k,
                                 case.scale)
    np.savez_compressed(HERE / "attention_cfg1.npz", row_sum=out.sum(-1).numpy(),
                        row_sq=(out * out).sum(-1).numpy(), rows=out[::19].numpy(),
                        cu_q=case.cu_q, cu_k=case.cu_k)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the VLCache reference checkout")
    ap.add_argument("--only", default=None, choices=["decode", "mrope", "rope", "attention"],
                    help="regenerate one fixture family only")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    if args.only:
        {"decode": run_decode_scenario, "mrope": run_mrope_cfg1, "rope": run_rope,
         "attention": run_attention_cfg1}[args.only]()
        return
    # BASELINE config 2 shape: 20 + 10,549 (77x137) + 48, ratio 0.1; cold copy at prefix 12
    run_metadata_scenario("cfg2", cold_prefix=12, warm_specs=[(20, 77 * 137, 48, True)], ratio=0.1)
    # config 1 shape under the reference rule R = ceil(0.1 * 1024) = 103
    run_metadata_scenario("cfg1", cold_prefix=16, warm_specs=[(16, 1024, 32, True)], ratio=0.1, seed=1)
    # mixed batch: text-only request + two warm requests at different offsets (config 3 style)
    run_metadata_scenario("mixed", cold_prefix=3, warm_specs=[(300, 2691, 0, False), (100, 2691, 40, True),
                                                              (511, 2691, 128, True)], ratio=0.05, seed=2)
    run_decode_scenario()
    run_mrope_cfg1()
    run_rope()
    run_attention_cfg1()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
