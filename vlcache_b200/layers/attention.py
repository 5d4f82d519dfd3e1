"""Attention layer, drop-in for nanovllm/layers/attention.py:1-75.

``Attention(num_heads, head_dim, scale, num_kv_heads)`` with ``k_cache``/``v_cache``
attributes injected by the model runner, and ``forward(q, k, v)`` reading the
per-step metadata from the global context, exactly like the reference.  The three
device steps run in this library's sm_100a kernels instead of Triton/flash-attn:
  * ``store_kvcache``  (reference :10-40, Triton)      -> vlc_store_kvcache
  * prefill            (reference :64-70, flash-attn)  -> vlc_prefill_attn (tcgen05)
  * decode             (reference :71-74, flash-attn)  -> vlc_decode_attn (split-K)
Optionally ``forward(q, k, v, positions=..., rotary_emb=...)`` takes q/k before RoPE
and rotates them in the scatter launch (vlc_rope_store_kvcache): the caller's
``q, k = self.rotary_emb(positions, q, k); o = self.attn(q, k, v)``
(nanovllm/models/qwen3.py:84-86) becomes one call with the same result.
``forward(q, None, None)`` attends over a cache that already holds this step's K/V
(stored by ``layers.linear.QKVParallelLinear.forward_rope_store``, which fuses the
QKV projection, RoPE and the scatter).
"""
from __future__ import annotations

import numpy as np
import torch
from torch import nn

from .. import ops
from ..utils.context import Context, get_context


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor):
    """Scatter new K/V rows into the paged cache by slot (-1 skipped).  Bit-exact copy."""
    ops.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


def _prefill_plan(context: Context, num_heads: int, num_kv_heads: int, device: torch.device) -> ops.PrefillPlan:
    """Plan once per step and cache it on the context (every layer shares it)."""
    plan = context.prefill_plan
    if plan is None:
        cq = context.cu_seqlens_q_host
        ck = context.cu_seqlens_k_host
        if cq is None:
            cq = context.cu_seqlens_q.cpu().numpy()   # device read: callers can avoid it
        if ck is None:
            ck = context.cu_seqlens_k.cpu().numpy()
        plan = ops.build_prefill_plan(np.asarray(cq), np.asarray(ck), num_heads, num_kv_heads,
                                      device=device)
        context.prefill_plan = plan
    elif plan.dev is None or plan.dev.device != device:
        plan.dev = torch.from_numpy(plan.host).to(device)
    return plan


def _workspace(context: Context, nbytes: int, device: torch.device) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    ws = context.workspace
    if ws is None or ws.numel() < nbytes or ws.device != device:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        context.workspace = ws
    return ws


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.layer_id = None  # set by engine.kv_cache.allocate_kv_cache (or the caller)

    def forward(self, q: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
                positions: torch.Tensor | None = None, rotary_emb: nn.Module | None = None):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if k is None or v is None:   # K/V already stored for this step (fused QKV projection)
            assert k is None and v is None and rotary_emb is None
            assert k_cache.numel() and v_cache.numel() and (context.block_tables is not None or
                                                            not context.is_prefill), \
                "attention without K/V reads them from the paged cache"
        if context.kv_ready is not None:    # this layer's reused rows are placed
            # (waited before the scatter: the attention kernel stays the scatter's direct
            # successor in the stream, so its programmatic launch overlaps the scatter)
            assert self.layer_id is not None, "kv_ready needs Attention.layer_id"
            torch.cuda.current_stream().wait_event(context.kv_ready[self.layer_id])
        have_cache = bool(k_cache.numel() and v_cache.numel()) and k is not None
        if rotary_emb is not None:
            assert positions is not None, "rotary_emb needs the positions"
            if have_cache and (context.block_tables is not None or not context.is_prefill):
                # K/V are read back from the cache: rotate and scatter in one launch
                q = ops.rope_store_kvcache(positions, q, k, v, rotary_emb.cos_sin_cache, k_cache, v_cache,
                                           context.slot_mapping)
                have_cache = False  # stored
            else:                   # cold prefill reads the in-flight K: rotate it too
                q, k = rotary_emb(positions, q, k)
        stored_plain = False  # k / v hold exactly the rows store_kvcache copied into the cache
        if have_cache:
            store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
            stored_plain = True
        if context.is_prefill:
            plan = _prefill_plan(context, self.num_heads, self.num_kv_heads, q.device)
            ws = _workspace(context, plan.workspace_bytes, q.device)
            if context.block_tables is not None:    # prefix cache / warm request: paged K/V
                # k / v (when given) are the rows just stored: self-attention sequences read
                # them directly and do not wait for the scatter
                inflight = k is not None and stored_plain
                o = ops.prefill_attention(q, k_cache, v_cache, context.block_tables, plan, self.scale,
                                          workspace=ws, k_new=k if inflight else None,
                                          v_new=v if inflight else None)
            else:                                   # cold prefill: the in-flight K/V
                o = ops.prefill_attention(q, k, v, None, plan, self.scale, workspace=ws)
        else:    # decode
            max_len = context.max_context_len
            if max_len is None:
                max_len = context.block_tables.size(1) * k_cache.shape[1]
            ws = _workspace(context, ops.decode_workspace_bytes(q.shape[0], self.num_heads, self.num_kv_heads,
                                                                max_len), q.device)
            o = ops.decode_attention(q, k_cache, v_cache, context.block_tables, context.context_lens, max_len,
                                     self.scale, workspace=ws)
            o = o.unsqueeze(1)
        return o
