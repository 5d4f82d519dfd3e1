"""Per-step attention metadata, drop-in for nanovllm/utils/context.py:1-27.

Same global-context API (``get_context`` / ``set_context`` / ``reset_context``) and the
same positional fields.  Added keyword-only fields (all optional, so existing callers
keep working):
  * ``prefill_plan``    — the host-built work plan of the prefill kernel (built lazily
                          from ``cu_seqlens_*`` on first use when the caller gives none,
                          then shared by every layer of the step);
  * ``cu_seqlens_q_host`` / ``cu_seqlens_k_host`` — host copies that let the plan be
                          built without a device-to-host read;
  * ``max_context_len`` — host-side bound for the decode grid (defaults to the
                          block-table width times the block size: no device read);
  * ``workspace``       — scratch tensor reused by every layer of the step;
  * ``kv_ready``        — per-layer CUDA events (``engine.kv_cache.copy_image_kv_per_layer``):
                          layer i's attention waits for event i before it reads the cache.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None
    # additions (keyword-only in set_context)
    prefill_plan: Any = None
    cu_seqlens_q_host: Any = None
    cu_seqlens_k_host: Any = None
    max_context_len: int | None = None
    workspace: torch.Tensor | None = None
    kv_ready: Any = None


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None, *, prefill_plan=None,
                cu_seqlens_q_host=None, cu_seqlens_k_host=None, max_context_len=None, workspace=None,
                kv_ready=None):
    global _CONTEXT
    _CONTEXT = Context(is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping,
                       context_lens, block_tables, prefill_plan, cu_seqlens_q_host, cu_seqlens_k_host,
                       max_context_len, workspace, kv_ready)


def reset_context():
    global _CONTEXT
    _CONTEXT = Context()
