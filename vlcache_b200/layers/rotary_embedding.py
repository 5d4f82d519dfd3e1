"""Rotary embeddings: nano-vllm's 1-D RoPE of new rows, and the M-RoPE position shift of
reused image K (the multimodal-RoPE path of the warm request).

``RotaryEmbedding`` / ``get_rope`` keep the interface of nanovllm/layers/rotary_embedding.py
(:17-48, :51-71): the same ``cos_sin_cache`` buffer, ``forward(positions, query, key)``
returning the rotated pair, computed by the vlc_rope_store_kvcache kernel.  The attention
layer can also take the rotation over and fuse it with the KV scatter
(``Attention.forward(q, k, v, positions=..., rotary_emb=...)``).

The reference (nanovllm/layers/rotary_embedding.py:51-60) ignores ``rope_scaling`` and
copies reused image K/V verbatim (nanovllm/engine/model_runner.py:170-180), which is
only right when the image keeps its position.  Qwen2.5-VL rotates vision keys with
multimodal RoPE (HF modeling_qwen2_5_vl.py:627-665): pair j of the rotate-half split
uses the t, h or w position of the token, by ``mrope_section`` = [16, 24, 24].  When a
cached image reappears at a different place in the prompt every vision position
moves by the same offset per section, and since R(p + d) = R(d) R(p) per pair the
cached K only needs one extra rotation by d.  ``MRopeShift`` applies it on the GPU
(vlc_mrope_shift), in place or while moving the rows to the new request's pages.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache

import torch
from torch import nn

from .. import ops


def rope_cos_sin_cache(rotary_dim: int, max_position: int, base: float) -> torch.Tensor:
    """[max_position, 1, rotary_dim] fp32: cos | sin of position x inv_freq.

    The table must hold the reference's values bit for bit (rotary_embedding.py:29-35:
    fp32 inv_freq = 1 / base^(2j/d), fp32 outer product with the positions, cos and sin
    by torch on the host), so it is built with the same torch operations in that order.
    """
    exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim
    inv_freq = 1.0 / (base ** exponents)
    angles = torch.outer(torch.arange(max_position, dtype=torch.float), inv_freq)
    return torch.cat((angles.cos(), angles.sin()), dim=-1).unsqueeze_(1)


class RotaryEmbedding(nn.Module):
    """Rotate-half RoPE, drop-in for nanovllm/layers/rotary_embedding.py:17-48."""

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float) -> None:
        super().__init__()
        self.head_size = head_size
        assert rotary_dim == head_size
        self.register_buffer("cos_sin_cache", rope_cos_sin_cache(rotary_dim, max_position_embeddings, base),
                             persistent=False)

    def forward(self, positions: torch.Tensor, query: torch.Tensor,
                key: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """query [N, H, D], key [N, Hk, D] bf16 and int64 positions [N] -> new rotated tensors."""
        return ops.rotary_embedding(positions, query, key, self.cos_sin_cache)


def get_rope(head_size: int, rotary_dim: int, max_position: int, base: float, rope_scaling: dict | None = None):
    """Shared instance per configuration; ``rope_scaling`` is ignored as in the reference
    (rotary_embedding.py:51-71: Qwen2.5-VL's M-RoPE sections are not applied to new rows)."""
    return _rope_cached(head_size, rotary_dim, max_position, base)


@lru_cache(1)
def _rope_cached(head_size: int, rotary_dim: int, max_position: int, base: float) -> RotaryEmbedding:
    return RotaryEmbedding(head_size, rotary_dim, max_position, base)


def image_position_delta(old_start: int, new_start: int, time_interval: int = 1) -> tuple[int, int, int]:
    """(dt, dh, dw) when an image's first vision position moves from ``old_start`` to
    ``new_start``: t = start * time_interval, h = start + row, w = start + col
    (HF modeling_qwen2_5_vl.py:1010-1020), so every section moves by the start offset."""
    d = int(new_start) - int(old_start)
    return (d * time_interval, d, d)


@dataclass
class MRopeShift:
    """Configuration of the shift: Qwen2.5-VL defaults (theta 1e6, sections 16/24/24)."""
    rope_theta: float = 1e6
    mrope_section: tuple[int, int, int] = (16, 24, 24)

    def shift_layer(self, k_cache: torch.Tensor, v_cache: torch.Tensor | None, src_slots: torch.Tensor,
                    dst_slots: torch.Tensor | None, delta_thw) -> None:
        """One layer; in place when ``dst_slots`` is None."""
        ops.mrope_shift(k_cache, v_cache, src_slots, dst_slots, delta_thw, self.mrope_section, self.rope_theta)

    def shift_all_layers(self, kv_cache: torch.Tensor, src_slots: torch.Tensor, dst_slots: torch.Tensor | None,
                         delta_thw) -> None:
        """Every layer of a ``[2, L, NB, BS, Hk, D]`` cache in one launch."""
        ops.mrope_shift_all_layers(kv_cache, src_slots, dst_slots, delta_thw, self.mrope_section, self.rope_theta)
