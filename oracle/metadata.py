"""Integer restatement of the reference's warm-prefill metadata (test oracle).

Follows, function by function:
  * ``ModelRunner._compute_slots``   nanovllm/engine/model_runner.py:160-168
  * ``ModelRunner.prepare_prefill``  nanovllm/engine/model_runner.py:194-320
    (warm branch :232-276, normal branch :278-291, block tables :182-186)
  * ``LLMEngine._do_image_kv_copy``  nanovllm/engine/llm_engine.py:58-89
  * ``BlockManager.try_partial_recompute`` R = ceil(ratio * N)
                                     nanovllm/engine/block_manager.py:56-75
  * ``ModelRunner.prepare_decode``   nanovllm/engine/model_runner.py:322-338
All arithmetic is vectorised numpy int64 -> int32 (bit-exact target).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def recompute_count(ratio: float, num_image_tokens: int) -> int:
    """R = ceil(ratio * N)  (block_manager.py:72)."""
    return int(math.ceil(ratio * num_image_tokens))


def compute_slots(block_table, start: int, end: int, block_size: int = 256) -> np.ndarray:
    """slot(p) = block_table[p // bs] * bs + p % bs for p in [start, end)  (model_runner.py:160-168)."""
    bt = np.asarray(block_table, dtype=np.int64)
    p = np.arange(start, end, dtype=np.int64)
    return (bt[p // block_size] * block_size + p % block_size).astype(np.int32)


@dataclass
class SeqSpec:
    """One request as the model runner sees it."""
    seqlen: int
    block_table: list[int]
    img_start: int | None = None     # image token range [img_start, img_end)
    img_end: int | None = None
    num_recompute: int = 0           # R; > 0 marks a warm (partial-recompute) request
    partial: bool = False


@dataclass
class PrefillMeta:
    positions: np.ndarray
    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    max_seqlen_q: int
    max_seqlen_k: int
    slot_mapping: np.ndarray
    block_tables: np.ndarray | None
    logit_indices: list[int] | None
    token_index: np.ndarray = field(default_factory=lambda: np.zeros(0, np.int64))  # which seq token each q row is


def prepare_prefill(seqs: list[SeqSpec], block_size: int = 256) -> PrefillMeta:
    """Warm requests become two virtual sub-sequences sharing the block table
    (model_runner.py:232-276): sub-seq 1 = tokens [0, img_start+R) attending to
    themselves, sub-seq 2 = tokens [img_end, n) attending to [0, n)."""
    positions, cu_q, cu_k, slots, vbt, tok_idx = [], [0], [0], [], [], []
    max_q = max_k = 0
    logit_indices: list[int] = []
    vidx = 0
    any_partial = False
    for s in seqs:
        n = s.seqlen
        if s.partial:
            any_partial = True
            a = s.img_start + s.num_recompute
            q1, k1 = a, a
            q2, k2 = n - s.img_end, n
            positions.append(np.arange(0, a))
            positions.append(np.arange(s.img_end, n))
            tok_idx.append(np.arange(0, a))
            tok_idx.append(np.arange(s.img_end, n))
            cu_q += [cu_q[-1] + q1, cu_q[-1] + q1 + q2]
            cu_k += [cu_k[-1] + k1, cu_k[-1] + k1 + k2]
            max_q = max(max_q, q1, q2)
            max_k = max(max_k, k1, k2)
            if s.block_table:
                slots.append(compute_slots(s.block_table, 0, a, block_size))
                slots.append(compute_slots(s.block_table, s.img_end, n, block_size))
                vbt += [list(s.block_table), list(s.block_table)]
            logit_indices.append(vidx + 1)
            vidx += 2
        else:
            positions.append(np.arange(0, n))
            tok_idx.append(np.arange(0, n))
            cu_q.append(cu_q[-1] + n)
            cu_k.append(cu_k[-1] + n)
            max_q = max(max_q, n)
            max_k = max(max_k, n)
            if s.block_table:
                slots.append(compute_slots(s.block_table, 0, n, block_size))
                vbt.append(list(s.block_table))
            logit_indices.append(vidx)
            vidx += 1
    block_tables = None
    if any_partial and vbt:
        width = max(len(b) for b in vbt)
        block_tables = np.array([b + [-1] * (width - len(b)) for b in vbt], dtype=np.int32)
    return PrefillMeta(
        positions=np.concatenate(positions).astype(np.int64) if positions else np.zeros(0, np.int64),
        cu_seqlens_q=np.asarray(cu_q, dtype=np.int32),
        cu_seqlens_k=np.asarray(cu_k, dtype=np.int32),
        max_seqlen_q=int(max_q),
        max_seqlen_k=int(max_k),
        slot_mapping=np.concatenate(slots).astype(np.int32) if slots else np.zeros(0, np.int32),
        block_tables=block_tables,
        logit_indices=logit_indices if any_partial else None,
        token_index=np.concatenate(tok_idx).astype(np.int64) if tok_idx else np.zeros(0, np.int64),
    )


def image_kv_copy_slots(img_start: int, img_end: int, num_recompute: int, new_block_table,
                        entry_img_start: int, entry_block_table, block_size: int = 256):
    """Old/new slots of the reused image rows [img_start+R, img_end)  (llm_engine.py:58-89)."""
    p = np.arange(img_start + num_recompute, img_end, dtype=np.int64)
    old_p = entry_img_start + (p - img_start)
    ebt = np.asarray(entry_block_table, dtype=np.int64)
    nbt = np.asarray(new_block_table, dtype=np.int64)
    old = ebt[old_p // block_size] * block_size + old_p % block_size
    new = nbt[p // block_size] * block_size + p % block_size
    return old.astype(np.int32), new.astype(np.int32)


def prepare_decode(seqlens, block_tables, block_size: int = 256):
    """Decode metadata (model_runner.py:322-338): positions, slot of the last token,
    context_lens, block tables padded with -1."""
    seqlens = np.asarray(seqlens, dtype=np.int64)
    pos = seqlens - 1
    last_block_num = seqlens - ((seqlens + block_size - 1) // block_size - 1) * block_size
    last_page = np.array([bt[-1] for bt in block_tables], dtype=np.int64)
    slot = last_page * block_size + last_block_num - 1
    width = max(len(b) for b in block_tables)
    bt = np.array([list(b) + [-1] * (width - len(b)) for b in block_tables], dtype=np.int32)
    return pos, slot.astype(np.int32), seqlens.astype(np.int32), bt
