"""fp32 attention restatement over a paged KV cache (test oracle, torch CPU).

Semantics of nanovllm/layers/attention.py:59-75:
  * prefill: ``flash_attn_varlen_func(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k,
    ..., causal=True, block_table=block_tables)`` — keys of sequence b are the first
    k_len_b slots of its block table; causal alignment is bottom-right, so query row i
    of b sees keys j <= k_len_b - q_len_b + i (flash-attn 2.8.3 flash_attn_interface.py,
    causal docstring);
  * decode: ``flash_attn_with_kvcache(q[:, None], k_cache, v_cache, cache_seqlens,
    block_table, causal=True)`` — the single query sees keys [0, len).
GQA: query head h uses KV head h // (H / Hk).  Softmax in fp32.
"""
from __future__ import annotations

import numpy as np
import torch


def gather_pages(cache: torch.Tensor, block_table, n: int) -> torch.Tensor:
    """First n keys of a sequence from a [num_blocks, block_size, Hk, D] cache."""
    bs = cache.shape[1]
    bt = torch.as_tensor(np.asarray(block_table)[: (n + bs - 1) // bs], dtype=torch.long)
    return cache[bt].reshape(-1, cache.shape[2], cache.shape[3])[:n]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, scale: float) -> torch.Tensor:
    """q [Nq, H, D], k/v [Nk, Hk, D] fp32; row i sees keys j <= q_pos[i]."""
    H, Hk = q.shape[1], k.shape[1]
    G = H // Hk
    kk = k.repeat_interleave(G, dim=1).permute(1, 2, 0)   # [H, D, Nk]
    vv = v.repeat_interleave(G, dim=1).permute(1, 0, 2)   # [H, Nk, D]
    qq = q.permute(1, 0, 2)                               # [H, Nq, D]
    s = torch.bmm(qq, kk) * scale                         # [H, Nq, Nk]
    j = torch.arange(k.shape[0])
    mask = j[None, :] > q_pos[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return torch.bmm(p, vv).permute(1, 0, 2)              # [Nq, H, D]


def varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, scale: float, causal: bool = False) -> torch.Tensor:
    """``flash_attn_varlen_func`` on contiguous-by-token q [total_q, H, d] and k / v
    [total_k, Hk, d]: sequence b's rows attend to its keys, every key when not causal (the
    vision tower's window and full attention, nanovllm/models/qwen2_5_vl.py:202-211),
    bottom-right causal otherwise.  fp32."""
    q = torch.as_tensor(q).float()
    k = torch.as_tensor(k).float()
    v = torch.as_tensor(v).float()
    cq = np.asarray(cu_seqlens_q)
    ck = np.asarray(cu_seqlens_k)
    out = torch.zeros_like(q)
    for b in range(len(cq) - 1):
        ql, kl = int(cq[b + 1] - cq[b]), int(ck[b + 1] - ck[b])
        if ql == 0:
            continue
        pos = torch.arange(kl - ql, kl) if causal else torch.full((ql,), kl - 1)
        out[cq[b]:cq[b + 1]] = _attend(q[cq[b]:cq[b + 1]], k[ck[b]:ck[b + 1]], v[ck[b]:ck[b + 1]], pos, scale)
    return out


def prefill_attention(q, k_cache, v_cache, block_tables, cu_seqlens_q, cu_seqlens_k, scale: float) -> torch.Tensor:
    q = torch.as_tensor(q).float()
    k_cache = torch.as_tensor(k_cache).float()
    v_cache = torch.as_tensor(v_cache).float()
    cq = np.asarray(cu_seqlens_q)
    ck = np.asarray(cu_seqlens_k)
    bts = np.asarray(block_tables)
    out = torch.zeros_like(q)
    for b in range(len(cq) - 1):
        ql, kl = int(cq[b + 1] - cq[b]), int(ck[b + 1] - ck[b])
        if ql == 0:
            continue
        k = gather_pages(k_cache, bts[b], kl)
        v = gather_pages(v_cache, bts[b], kl)
        pos = torch.arange(kl - ql, kl)
        out[cq[b]:cq[b + 1]] = _attend(q[cq[b]:cq[b + 1]], k, v, pos, scale)
    return out


def prefill_attention_rows(q, k_cache, v_cache, block_tables, cu_seqlens_q, cu_seqlens_k, scale: float,
                           rows) -> torch.Tensor:
    """The rows ``rows`` (absolute query indices) of ``prefill_attention``, computed alone:
    row i of sequence b sees keys j <= k_len_b - q_len_b + (i - cu_q[b]), as above.  Lets a
    test check a sample of a problem whose full fp32 evaluation would not fit the host."""
    q = torch.as_tensor(q).float()
    k_cache = torch.as_tensor(k_cache).float()
    v_cache = torch.as_tensor(v_cache).float()
    cq = np.asarray(cu_seqlens_q)
    ck = np.asarray(cu_seqlens_k)
    bts = np.asarray(block_tables)
    rows = np.asarray(rows, dtype=np.int64)
    seq = np.searchsorted(cq, rows, side="right") - 1
    out = torch.zeros(len(rows), q.shape[1], q.shape[2])
    for b in np.unique(seq):
        sel = np.nonzero(seq == b)[0]
        ql, kl = int(cq[b + 1] - cq[b]), int(ck[b + 1] - ck[b])
        k = gather_pages(k_cache, bts[b], kl)
        v = gather_pages(v_cache, bts[b], kl)
        pos = torch.as_tensor(kl - ql + (rows[sel] - cq[b]))
        out[sel] = _attend(q[rows[sel]], k, v, pos, scale)
    return out


def decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale: float) -> torch.Tensor:
    q = torch.as_tensor(q).float()
    if q.dim() == 4:
        q = q[:, 0]
    k_cache = torch.as_tensor(k_cache).float()
    v_cache = torch.as_tensor(v_cache).float()
    lens = np.asarray(context_lens)
    bts = np.asarray(block_tables)
    out = torch.zeros_like(q)
    for b in range(q.shape[0]):
        n = int(lens[b])
        if n <= 0:
            continue
        k = gather_pages(k_cache, bts[b], n)
        v = gather_pages(v_cache, bts[b], n)
        out[b:b + 1] = _attend(q[b:b + 1], k, v, torch.tensor([n - 1]), scale)
    return out


def causal_pairs(cu_seqlens_q, cu_seqlens_k) -> int:
    """Sum over query rows of visible keys (per head): the algorithmic work unit."""
    cq = np.asarray(cu_seqlens_q, dtype=np.int64)
    ck = np.asarray(cu_seqlens_k, dtype=np.int64)
    tot = 0
    for b in range(len(cq) - 1):
        ql, kl = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
        first = kl - ql + 1
        tot += (first + kl) * ql // 2
    return int(tot)
