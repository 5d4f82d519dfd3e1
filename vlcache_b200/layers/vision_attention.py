"""Varlen attention of the vision tower, drop-in for the flash-attn call in
nanovllm/models/qwen2_5_vl.py:202-211 (``VisionAttention.forward``).

The Qwen2.5-VL vision transformer runs ``flash_attn_varlen_func(q, k, v, cu_seqlens,
cu_seqlens, max_seqlen, max_seqlen, causal=False)`` over contiguous ``[tokens, heads, 80]``
q/k/v: window attention (``cu_window_seqlens``, windows of about 64 patches,
qwen2_5_vl.py:392-435) in most blocks and full attention over the image in the
``fullatt_block_indexes`` blocks.  ``varlen_attention`` takes the same arguments and runs
this library's tcgen05 attention kernel with a non-causal plan (head dims 80..128: the
kernel zero-pads tiles to 128 columns on load and writes the real ones).  The plan is
built on the host from ``cu_seqlens``; pass ``cu_seqlens_host`` (or a ``plan``) when the
caller has it, else one device read plans the launch, as the reference's
``max_seqlen = (...).max().item()`` already reads the device.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops


def plan_varlen(cu_seqlens_q, cu_seqlens_k, num_heads: int, num_kv_heads: int, head_dim: int, causal: bool = False,
                device=None) -> ops.PrefillPlan:
    """Work plan of one varlen attention launch from host cu_seqlens (reusable by every
    layer with the same sequences, e.g. all window-attention blocks of one image)."""
    return ops.build_prefill_plan(np.asarray(cu_seqlens_q), np.asarray(cu_seqlens_k), num_heads, num_kv_heads,
                                  head_dim, device=device, causal=causal)


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                     cu_seqlens_k: torch.Tensor, max_seqlen_q: int | None = None, max_seqlen_k: int | None = None,
                     softmax_scale: float | None = None, causal: bool = False, *, cu_seqlens_q_host=None,
                     cu_seqlens_k_host=None, plan: ops.PrefillPlan | None = None, out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """``flash_attn_varlen_func`` semantics for contiguous-by-token q ``[total_q, H, d]`` and
    k / v ``[total_k, Hk, d]`` (any token stride): softmax(scale q k^T) v per sequence,
    causal with bottom-right alignment or not; ``softmax_scale`` defaults to d^-1/2."""
    H, d = q.shape[1], q.shape[2]
    Hk = k.shape[1]
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(d)
    if plan is None:
        cq = cu_seqlens_q_host if cu_seqlens_q_host is not None else cu_seqlens_q.cpu().numpy()
        ck = cu_seqlens_k_host if cu_seqlens_k_host is not None else (
            cq if cu_seqlens_k is cu_seqlens_q else cu_seqlens_k.cpu().numpy())
        plan = plan_varlen(cq, ck, H, Hk, d, causal, device=q.device)
    return ops.prefill_attention(q, k, v, None, plan, softmax_scale, out=out, workspace=workspace)
