"""M-RoPE restatement (test oracle, torch fp32 / numpy).

The reference LLM applies 1-D rotate-half RoPE (nanovllm/layers/rotary_embedding.py:6-14,
29-48) and drops ``rope_scaling``; Qwen2.5-VL's multimodal RoPE is therefore taken
from HF transformers 5.5.0 models/qwen2_5_vl/modeling_qwen2_5_vl.py:
  * ``rotate_half``                       :149-153
  * ``Qwen2_5_VLRotaryEmbedding``        :545-610 (inv_freq, fp32 freqs, cat(freqs, freqs))
  * ``apply_multimodal_rotary_pos_emb``   :627-665 (sections [t, h, w] over the pairs)
  * ``get_vision_position_ids``           :968-1022 (t = st, h = st + row, w = st + col)
The shift restatement ``shift_rows`` is the same rotation the position-shift kernel
applies: R(a + d) = R(d) R(a) per rotate-half pair, with a host-built fp32 cos/sin
table for the per-section delta and single-rounded fp32 products.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import math

import numpy as np
import torch


def inv_freq(head_dim: int = 128, theta: float = 1e6) -> torch.Tensor:
    """1 / theta^(arange(0, d, 2) / d) in fp32 (modeling_qwen2_5_vl.py:589-591)."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim))


def vision_positions(start: int, grid_h: int, grid_w: int, grid_t: int = 1) -> np.ndarray:
    """[3, N] (t, h, w) positions of a merged vision grid starting at ``start``
    (modeling_qwen2_5_vl.py:1010-1020)."""
    w = np.tile(np.arange(start, start + grid_w), grid_h * grid_t)
    h = np.repeat(np.arange(start, start + grid_h), grid_w * grid_t)
    t = np.full(grid_h * grid_w * grid_t, start)
    return np.stack([t, h, w]).astype(np.int64)


def text_positions(start: int, n: int) -> np.ndarray:
    p = np.arange(start, start + n, dtype=np.int64)
    return np.stack([p, p, p])


def mrope_cos_sin(pos_thw: np.ndarray, sections=(16, 24, 24), head_dim: int = 128, theta: float = 1e6):
    """cos/sin [N, head_dim] with the per-section position selection (fp32)."""
    inv = inv_freq(head_dim, theta)
    pos = torch.as_tensor(pos_thw, dtype=torch.float32)                     # [3, N]
    freqs = pos[:, :, None] * inv[None, None, :]                            # [3, N, d/2]
    emb = torch.cat([freqs, freqs], dim=-1)                                 # [3, N, d]
    cos, sin = emb.cos(), emb.sin()
    sec2 = list(sections) * 2
    cos = torch.cat([m[i % 3] for i, m in enumerate(cos.split(sec2, dim=-1))], dim=-1)
    sin = torch.cat([m[i % 3] for i, m in enumerate(sin.split(sec2, dim=-1))], dim=-1)
    return cos, sin


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_mrope(x: torch.Tensor, pos_thw: np.ndarray, sections=(16, 24, 24), theta: float = 1e6) -> torch.Tensor:
    """x [N, heads, d] (fp32) rotated at positions pos_thw [3, N]."""
    cos, sin = mrope_cos_sin(pos_thw, sections, x.shape[-1], theta)
    cos, sin = cos[:, None, :], sin[:, None, :]
    return x * cos + rotate_half(x) * sin


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]


def _inv_freq_like_kernel(j: int, head_dim: int, theta: float) -> np.float32:
    """fp32 inv_freq[j] = 1 / powf(theta, float(2j) / float(d)) with the C library's powf,
    so the table matches the one the kernel's host code builds bit for bit."""
    e = np.float32(2 * j) / np.float32(head_dim)
    p = np.float32(_libm.powf(float(np.float32(theta)), float(e)))
    return np.float32(np.float32(1.0) / p)


def shift_table(delta_thw, sections=(16, 24, 24), head_dim: int = 128, theta: float = 1e6):
    """fp32 cos/sin of inv_freq[j] * delta_sec(j) for the rotate-half pairs."""
    half = head_dim // 2
    c = np.zeros(half, np.float32)
    s = np.zeros(half, np.float32)
    for j in range(half):
        sec = 0 if j < sections[0] else (1 if j < sections[0] + sections[1] else 2)
        a = float(_inv_freq_like_kernel(j, head_dim, theta)) * float(delta_thw[sec])
        c[j] = np.float32(math.cos(a))
        s[j] = np.float32(math.sin(a))
    return c, s


def shift_rows(k_bits: np.ndarray, delta_thw, sections=(16, 24, 24), theta: float = 1e6) -> np.ndarray:
    """Rotate bf16 rows k_bits [n, heads, d] (uint16) by the delta; returns bf16 bits.

    y1 = fma(x1, c, -(x2*s)),  y2 = fma(x2, c, x1*s)  with single-rounded fp32 products.
    """
    d = k_bits.shape[-1]
    half = d // 2
    c, s = shift_table(delta_thw, sections, d, theta)
    x = bf16_bits_to_f32(k_bits).astype(np.float64)
    x1, x2 = x[..., :half], x[..., half:]
    t1 = (x2 * s).astype(np.float32).astype(np.float64)
    t2 = (x1 * s).astype(np.float32).astype(np.float64)
    y1 = (x1 * c - t1).astype(np.float32)
    y2 = (x2 * c + t2).astype(np.float32)
    return f32_to_bf16_bits(np.concatenate([y1, y2], axis=-1))
