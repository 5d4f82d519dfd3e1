"""KV-cache allocation, reused-image KV placement and warm-prefill metadata.

Host side of the hot path, mirroring nano-vllm's model runner / engine:
  * ``allocate_kv_cache``     — nanovllm/engine/model_runner.py:127-158: one tensor
    ``[2, L, num_blocks, block_size, Hk, D]`` whose per-layer views are handed to every
    module with ``k_cache``/``v_cache``;
  * ``copy_image_kv``         — model_runner.py:170-180 + llm_engine.py:58-89: move the
    reused image rows of every layer to the new request's pages, re-rotating K by the
    M-RoPE position delta (one launch for all layers);
  * ``WarmPrefillBuilder``    — model_runner.py:160-168 (``_compute_slots``) and
    :194-320 (``prepare_prefill``, warm branch :232-276): cu_seqlens, slot_mapping,
    padded block tables, positions, vectorised, plus the attention plan, all built from
    host data so no device read is needed during the step;
  * ``prepare_decode``        — model_runner.py:322-338.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..layers.rotary_embedding import MRopeShift
from ..utils.context import set_context

BLOCK_SIZE = 256


def allocate_kv_cache(model: torch.nn.Module | None, num_layers: int, num_blocks: int, num_kv_heads: int,
                      head_dim: int = 128, block_size: int = BLOCK_SIZE, dtype=torch.bfloat16,
                      device="cuda") -> torch.Tensor:
    kv_cache = torch.empty(2, num_layers, num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype,
                           device=device)
    if model is not None:
        layer_id = 0
        for module in model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                module.k_cache = kv_cache[0, layer_id]
                module.v_cache = kv_cache[1, layer_id]
                layer_id += 1
    return kv_cache


def compute_slots(block_table, start: int, end: int, block_size: int = BLOCK_SIZE) -> np.ndarray:
    """slot(p) = block_table[p // block_size] * block_size + p % block_size, p in [start, end)."""
    bt = np.asarray(block_table, dtype=np.int64)
    p = np.arange(start, end, dtype=np.int64)
    return (bt[p // block_size] * block_size + p % block_size).astype(np.int32)


def image_reuse_slots(img_start: int, img_end: int, num_recompute: int, new_block_table, old_img_start: int,
                      old_block_table, block_size: int = BLOCK_SIZE):
    """Source/destination slots of the reused image rows [img_start + R, img_end)."""
    p = np.arange(img_start + num_recompute, img_end, dtype=np.int64)
    old_p = old_img_start + (p - img_start)
    obt = np.asarray(old_block_table, dtype=np.int64)
    nbt = np.asarray(new_block_table, dtype=np.int64)
    src = obt[old_p // block_size] * block_size + old_p % block_size
    dst = nbt[p // block_size] * block_size + p % block_size
    return src.astype(np.int32), dst.astype(np.int32)


def copy_image_kv(kv_cache: torch.Tensor, old_slots, new_slots, delta_thw=(0, 0, 0),
                  shift: MRopeShift | None = None) -> None:
    """Move reused image K/V rows (all layers) to new slots, rotating K by ``delta_thw``.

    With a zero delta this is the reference's verbatim copy.  old and new slot sets
    must be disjoint (they are: the new request owns freshly allocated pages)."""
    if len(old_slots) == 0:
        return
    dev = kv_cache.device
    src = torch.as_tensor(np.asarray(old_slots, dtype=np.int32)).pin_memory().to(dev, non_blocking=True)
    dst = torch.as_tensor(np.asarray(new_slots, dtype=np.int32)).pin_memory().to(dev, non_blocking=True)
    (shift or MRopeShift()).shift_all_layers(kv_cache, src, dst, delta_thw)


@dataclass
class WarmRequest:
    """What the runner knows about one request at prefill time."""
    seqlen: int
    block_table: list[int]
    img_start: int | None = None
    img_end: int | None = None
    num_recompute: int = 0
    partial: bool = False


@dataclass
class PrefillBatch:
    positions: np.ndarray
    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    max_seqlen_q: int
    max_seqlen_k: int
    slot_mapping: np.ndarray
    block_tables: np.ndarray | None
    logit_indices: list[int] | None
    plan: ops.PrefillPlan | None = None
    device_tensors: dict = field(default_factory=dict)


def recompute_count(ratio: float, num_image_tokens: int) -> int:
    """R = ceil(ratio * N) (nanovllm/engine/block_manager.py:72)."""
    return int(math.ceil(ratio * num_image_tokens))


class WarmPrefillBuilder:
    """Vectorised ``prepare_prefill``: metadata for a batch of cold and warm requests."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int = 128, block_size: int = BLOCK_SIZE):
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size

    def build(self, reqs: list[WarmRequest]) -> PrefillBatch:
        bs = self.block_size
        pos, cq, ck, slots, vbt = [], [0], [0], [], []
        max_q = max_k = 0
        logit_indices: list[int] = []
        vidx = 0
        any_partial = False
        for r in reqs:
            n = r.seqlen
            if r.partial:
                any_partial = True
                a = r.img_start + r.num_recompute
                pos += [np.arange(0, a), np.arange(r.img_end, n)]
                cq += [cq[-1] + a, cq[-1] + a + (n - r.img_end)]
                ck += [ck[-1] + a, ck[-1] + a + n]
                max_q = max(max_q, a, n - r.img_end)
                max_k = max(max_k, a, n)
                if r.block_table:
                    slots += [compute_slots(r.block_table, 0, a, bs), compute_slots(r.block_table, r.img_end, n, bs)]
                    vbt += [r.block_table, r.block_table]
                logit_indices.append(vidx + 1)
                vidx += 2
            else:
                pos.append(np.arange(0, n))
                cq.append(cq[-1] + n)
                ck.append(ck[-1] + n)
                max_q, max_k = max(max_q, n), max(max_k, n)
                if r.block_table:
                    slots.append(compute_slots(r.block_table, 0, n, bs))
                    vbt.append(r.block_table)
                logit_indices.append(vidx)
                vidx += 1
        block_tables = None
        if any_partial and vbt:
            width = max(len(b) for b in vbt)
            block_tables = np.full((len(vbt), width), -1, dtype=np.int32)
            for i, b in enumerate(vbt):
                block_tables[i, :len(b)] = b
        cq_a = np.asarray(cq, dtype=np.int32)
        ck_a = np.asarray(ck, dtype=np.int32)
        return PrefillBatch(
            positions=np.concatenate(pos).astype(np.int64) if pos else np.zeros(0, np.int64),
            cu_seqlens_q=cq_a, cu_seqlens_k=ck_a, max_seqlen_q=max_q, max_seqlen_k=max_k,
            slot_mapping=np.concatenate(slots).astype(np.int32) if slots else np.zeros(0, np.int32),
            block_tables=block_tables, logit_indices=logit_indices if any_partial else None)

    def upload(self, batch: PrefillBatch, device="cuda") -> PrefillBatch:
        """Copy the metadata to the device (pinned, non-blocking), plan the attention
        kernel, and install everything with ``set_context``."""
        def up(a, dtype):
            return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).pin_memory().to(device, non_blocking=True)
        t = {
            "positions": up(batch.positions, torch.int64),
            "cu_seqlens_q": up(batch.cu_seqlens_q, torch.int32),
            "cu_seqlens_k": up(batch.cu_seqlens_k, torch.int32),
            "slot_mapping": up(batch.slot_mapping, torch.int32),
            "block_tables": None if batch.block_tables is None else up(batch.block_tables, torch.int32),
        }
        batch.plan = ops.build_prefill_plan(batch.cu_seqlens_q, batch.cu_seqlens_k, self.num_heads,
                                            self.num_kv_heads, self.head_dim, device=device)
        batch.device_tensors = t
        set_context(True, t["cu_seqlens_q"], t["cu_seqlens_k"], batch.max_seqlen_q, batch.max_seqlen_k,
                    t["slot_mapping"], None, t["block_tables"], prefill_plan=batch.plan,
                    cu_seqlens_q_host=batch.cu_seqlens_q, cu_seqlens_k_host=batch.cu_seqlens_k)
        return batch


def prepare_decode(seqlens, block_tables, block_size: int = BLOCK_SIZE, device="cuda"):
    """Decode metadata (model_runner.py:322-338) + ``set_context``; returns positions."""
    seqlens = np.asarray(seqlens, dtype=np.int64)
    last_n = seqlens - ((seqlens + block_size - 1) // block_size - 1) * block_size
    last_page = np.array([bt[-1] for bt in block_tables], dtype=np.int64)
    slot = (last_page * block_size + last_n - 1).astype(np.int32)
    width = max(len(b) for b in block_tables)
    bt = np.full((len(block_tables), width), -1, dtype=np.int32)
    for i, b in enumerate(block_tables):
        bt[i, :len(b)] = b

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).pin_memory().to(device, non_blocking=True)
    positions = up(seqlens - 1, torch.int64)
    set_context(False, slot_mapping=up(slot, torch.int32), context_lens=up(seqlens, torch.int32),
                block_tables=up(bt, torch.int32), max_context_len=int(width * block_size))
    return positions
