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


@dataclass
class CacheBudget:
    """Block counts ``allocate_kv_cache`` derives from the device's memory, as the
    reference's ``ModelRunner.allocate_kv_cache`` does (model_runner.py:130-151)."""
    num_kvcache_blocks: int
    num_encoder_blocks: int
    kv_block_bytes: int
    encoder_block_bytes: int
    available_bytes: float


def cache_budget(num_layers: int, num_kv_heads: int, head_dim: int, hidden_size: int, *, block_size: int = BLOCK_SIZE,
                 dtype=torch.bfloat16, gpu_memory_utilization: float = 0.9, encoder_cache_ratio: float = 0.2,
                 mem_info: tuple[int, int] | None = None, peak_bytes: int | None = None,
                 current_bytes: int | None = None) -> CacheBudget:
    """The reference's sizing rule (model_runner.py:130-151):
    ``available = total * gpu_memory_utilization - used - peak + current`` (used = total -
    free; peak / current = torch's allocated-bytes statistics), ``encoder_cache_ratio`` of
    it for the encoder cache (blocks of ``block_size`` tokens x ``hidden_size``), the rest
    for KV blocks of ``2 * layers * block_size * Hk * head_dim`` elements.  The memory
    figures default to the current device's; pass them to size for another budget."""
    if mem_info is None:
        free, total = torch.cuda.mem_get_info()
    else:
        free, total = mem_info
    if peak_bytes is None or current_bytes is None:
        stats = torch.cuda.memory_stats()
        peak_bytes = stats.get("allocated_bytes.all.peak", 0) if peak_bytes is None else peak_bytes
        current_bytes = stats.get("allocated_bytes.all.current", 0) if current_bytes is None else current_bytes
    itemsize = torch.empty((), dtype=dtype).element_size()
    used = total - free
    kv_block_bytes = 2 * num_layers * block_size * num_kv_heads * head_dim * itemsize
    encoder_block_bytes = block_size * hidden_size * itemsize
    available = total * gpu_memory_utilization - used - peak_bytes + current_bytes
    encoder_memory = available * encoder_cache_ratio
    kv_memory = available - encoder_memory
    budget = CacheBudget(int(kv_memory) // kv_block_bytes, int(encoder_memory) // encoder_block_bytes,
                         kv_block_bytes, encoder_block_bytes, available)
    if budget.num_kvcache_blocks <= 0:
        raise ValueError(f"no memory left for KV blocks ({available / 2**30:.2f} GiB available)")
    return budget


def allocate_kv_cache(model: torch.nn.Module | None, num_layers: int, num_blocks: int | None, num_kv_heads: int,
                      head_dim: int = 128, block_size: int = BLOCK_SIZE, dtype=torch.bfloat16,
                      device="cuda", *, hidden_size: int | None = None, gpu_memory_utilization: float = 0.9,
                      encoder_cache_ratio: float = 0.2) -> torch.Tensor:
    """``[2, L, num_blocks, block_size, Hk, D]`` with per-layer views handed to every module
    that has ``k_cache`` / ``v_cache`` (model_runner.py:152-158), plus the module's
    ``layer_id``.  ``num_blocks=None`` sizes the pool from the device's free memory with
    the reference's rule (``cache_budget``, which needs ``hidden_size`` for the encoder
    cache share); the tensor's ``budget`` attribute then holds the block counts, the
    encoder-cache block count included."""
    budget = None
    if num_blocks is None:
        if hidden_size is None:
            raise ValueError("sizing from free memory needs hidden_size (the encoder cache's share)")
        with torch.cuda.device(torch.device(device)):
            budget = cache_budget(num_layers, num_kv_heads, head_dim, hidden_size, block_size=block_size, dtype=dtype,
                                  gpu_memory_utilization=gpu_memory_utilization,
                                  encoder_cache_ratio=encoder_cache_ratio)
        num_blocks = budget.num_kvcache_blocks
    kv_cache = torch.empty(2, num_layers, num_blocks, block_size, num_kv_heads, head_dim, dtype=dtype,
                           device=device)
    kv_cache.budget = budget
    if model is not None:
        layer_id = 0
        for module in model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                module.k_cache = kv_cache[0, layer_id]
                module.v_cache = kv_cache[1, layer_id]
                module.layer_id = layer_id  # index into Context.kv_ready
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


def check_reuse_slots(old_slots, new_slots) -> None:
    """Raise ValueError when a slot is the source of one reused row and the destination
    of another.  The reference's ``flat[:, :, new] = flat[:, :, old]``
    (model_runner.py:180) reads every row before writing any; the shift kernel moves
    row by row, which gives the same result exactly when no destination is another
    row's source.  A row moved onto itself (a page shared by the old and the new block
    table at the same position) is allowed."""
    old = np.asarray(old_slots, dtype=np.int64).ravel()
    new = np.asarray(new_slots, dtype=np.int64).ravel()
    if old.shape != new.shape:
        raise ValueError("old and new slot lists differ in length")
    common, i_old, i_new = np.intersect1d(old, new, assume_unique=False, return_indices=True)
    if len(common) and np.any(i_old != i_new):
        bad = int(common[np.nonzero(i_old != i_new)[0][0]])
        raise ValueError(f"reused image slots overlap: slot {bad} is the source of one row and the "
                         "destination of another (old and new block tables share a page at "
                         "different positions); move the rows through a fresh page first")


def copy_image_kv(kv_cache: torch.Tensor, old_slots, new_slots, delta_thw=(0, 0, 0),
                  shift: MRopeShift | None = None) -> None:
    """Move reused image K/V rows (all layers) to new slots, rotating K by ``delta_thw``.

    With a zero delta this is the reference's verbatim copy.  No destination may be
    another row's source (``check_reuse_slots``, checked here on the host lists)."""
    if len(old_slots) == 0:
        return
    check_reuse_slots(old_slots, new_slots)
    dev = kv_cache.device
    src = torch.as_tensor(np.asarray(old_slots, dtype=np.int32)).pin_memory().to(dev, non_blocking=True)
    dst = torch.as_tensor(np.asarray(new_slots, dtype=np.int32)).pin_memory().to(dev, non_blocking=True)
    (shift or MRopeShift()).shift_all_layers(kv_cache, src, dst, delta_thw)


def copy_image_kv_per_layer(kv_cache: torch.Tensor, src_slots: torch.Tensor, dst_slots: torch.Tensor,
                            delta_thw=(0, 0, 0), stream: torch.cuda.Stream | None = None,
                            shift: MRopeShift | None = None, check: bool = False) -> list:
    """``copy_image_kv`` as one launch per layer on ``stream`` (device int32 slot tensors),
    returning one CUDA event per layer.  Pass the events as ``set_context(..., kv_ready=...)``:
    each attention layer waits only for its own layer's rows, so the re-placement of later
    layers overlaps the compute of earlier ones.  Give ``stream`` a lower priority than
    the compute stream (the layers' kernels then take the SMs first).  ``check=True`` runs
    ``check_reuse_slots`` on a host copy of the slots first (a device read: not for
    graph capture)."""
    if check:
        check_reuse_slots(src_slots.cpu().numpy(), dst_slots.cpu().numpy())
    sh = shift or MRopeShift()
    cur = torch.cuda.current_stream()
    stream = stream or cur
    stream.wait_stream(cur)
    events = []
    with torch.cuda.stream(stream):
        for layer in range(kv_cache.shape[1]):
            if src_slots.numel():
                sh.shift_layer(kv_cache[0, layer], kv_cache[1, layer], src_slots, dst_slots, delta_thw)
            ev = torch.cuda.Event()
            ev.record(stream)
            events.append(ev)
    if stream is not cur:
        src_slots.record_stream(stream)
        dst_slots.record_stream(stream)
    return events


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
class ImageReuse:
    """A warm request's reused image rows: where the image sat in the request that cached
    it (the encoder-cache entry's ``img_start`` and block table)."""
    request: int
    old_img_start: int
    old_block_table: list[int]


@dataclass
class PrefillBatch:
    positions: np.ndarray | None
    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    max_seqlen_q: int
    max_seqlen_k: int
    slot_mapping: np.ndarray | None
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

    def build_device(self, reqs: list[WarmRequest], reuse: list[ImageReuse] = (), device="cuda",
                     install: bool = True) -> PrefillBatch:
        """``build`` on the device: the same arrays, bit for bit, from O(requests) host work.

        The host lists one descriptor per virtual sequence (two per warm request) and per
        reused image, uploads them with the block tables in one pinned copy, and one
        kernel (vlc_warm_metadata) writes positions, slot_mapping, the padded block tables
        and the image-reuse source/destination slots.  With ``install`` the attention is
        planned and the context set, as ``upload`` does.  The device tensors are in
        ``device_tensors`` (``reuse_src`` / ``reuse_dst`` for the image move)."""
        vdesc, cq, ck, tables = [], [0], [0], []
        offsets, lengths = [], []
        q = slot = row = 0
        max_q = max_k = width = 0
        vidx = 0
        logit_indices: list[int] = []
        any_partial = False
        total = 0  # table entries so far (running offsets: O(requests))
        for r in reqs:
            offsets.append(total)
            lengths.append(len(r.block_table))
            total += lengths[-1]
            tables.extend(r.block_table)  # one flat list, converted once below
        for i, r in enumerate(reqs):
            n, L, off = r.seqlen, lengths[i], offsets[i]
            has = L > 0
            if r.partial:
                any_partial = True
                a = r.img_start + r.num_recompute
                parts = [(a, 0), (n - r.img_end, r.img_end)]
                cq += [cq[-1] + a, cq[-1] + a + (n - r.img_end)]
                ck += [ck[-1] + a, ck[-1] + a + n]
                max_q = max(max_q, a, n - r.img_end)
                max_k = max(max_k, a, n)
                logit_indices.append(vidx + 1)
                vidx += 2
            else:
                parts = [(n, 0)]
                cq.append(cq[-1] + n)
                ck.append(ck[-1] + n)
                max_q, max_k = max(max_q, n), max(max_k, n)
                logit_indices.append(vidx)
                vidx += 1
            for qlen, pos0 in parts:
                vdesc.append([q, qlen, pos0, off, L, slot if has else -1, row if has else -1])
                q += qlen
                if has:
                    slot += qlen
                    row += 1
                    width = max(width, L)
        rdesc, out = [], 0
        for it in reuse:
            r = reqs[it.request]
            count = r.img_end - r.img_start - r.num_recompute
            old_off = total  # after the requests' tables and the earlier old tables
            tables.extend(it.old_block_table)
            total += len(it.old_block_table)
            rdesc.append([out, count, r.img_start + r.num_recompute, offsets[it.request], lengths[it.request],
                          it.old_img_start + r.num_recompute, old_off, len(it.old_block_table)])
            out += count
        nv, nr = len(vdesc), len(rdesc)
        flat_tables = np.asarray(tables, dtype=np.int32)
        desc = np.concatenate([np.asarray(vdesc, np.int32).reshape(-1), np.asarray(rdesc, np.int32).reshape(-1),
                               flat_tables, np.zeros(1, np.int32)])
        desc_dev = torch.from_numpy(desc).pin_memory().to(device, non_blocking=True)
        rows = row if any_partial else 0
        positions, slots, bt, src, dst = ops.warm_metadata(
            desc_dev, nv, nv * ops.VSEQ_INTS, nr, nv * ops.VSEQ_INTS + nr * ops.REUSE_INTS, self.block_size, q,
            slot, rows, width if rows else 0, out)
        cq_a = np.asarray(cq, dtype=np.int32)
        ck_a = np.asarray(ck, dtype=np.int32)
        batch = PrefillBatch(positions=None, cu_seqlens_q=cq_a, cu_seqlens_k=ck_a, max_seqlen_q=max_q,
                             max_seqlen_k=max_k, slot_mapping=None, block_tables=None,
                             logit_indices=logit_indices if any_partial else None)
        batch.device_tensors = {
            "positions": positions, "slot_mapping": slots, "block_tables": bt, "reuse_src": src, "reuse_dst": dst,
            "cu_seqlens_q": torch.from_numpy(cq_a).pin_memory().to(device, non_blocking=True),
            "cu_seqlens_k": torch.from_numpy(ck_a).pin_memory().to(device, non_blocking=True),
            "descriptors": desc_dev,
        }
        if install:
            t = batch.device_tensors
            batch.plan = ops.build_prefill_plan(cq_a, ck_a, self.num_heads, self.num_kv_heads, self.head_dim,
                                                device=device)
            set_context(True, t["cu_seqlens_q"], t["cu_seqlens_k"], max_q, max_k, t["slot_mapping"], None,
                        t["block_tables"], prefill_plan=batch.plan, cu_seqlens_q_host=cq_a,
                        cu_seqlens_k_host=ck_a)
        return batch

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
