"""M-RoPE position shift for reused image K (the multimodal-RoPE path of the warm request).

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

import torch

from .. import ops


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
