"""CPU restatement of the rotary embedding + KV scatter of new rows (test oracle only).

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
use this module, as the checker; the product path never calls it.

It follows the reference's 1-D rotate-half RoPE and its KV store:
  * ``apply_rotary_emb``        nanovllm/layers/rotary_embedding.py:6-14 — x split in
    halves (x1, x2), y1 = x1*cos - x2*sin, y2 = x2*cos + x1*sin in fp32, cast to bf16;
  * ``RotaryEmbedding.forward`` rotary_embedding.py:37-48 — cos | sin gathered from
    ``cos_sin_cache[positions]``, the same rotation applied to query and key;
  * ``store_kvcache``           nanovllm/layers/attention.py:10-40 — the key and value
    rows written to cache row ``slot_mapping[i]``, slot -1 skipped.
numpy float32 arithmetic rounds every product, sum and difference on its own, as the
reference function evaluated op by op does.  The cos/sin table is an input (the
reference builds it with torch at :29-35); the golden fixture pins the table this
package builds against the reference's.
"""
from __future__ import annotations

import numpy as np

from .mrope import bf16_bits_to_f32, f32_to_bf16_bits


def rope_rows(x_bits: np.ndarray, positions: np.ndarray, cos_sin: np.ndarray) -> np.ndarray:
    """bf16 rows ``x_bits`` [N, heads, D] (uint16) rotated at ``positions`` [N] with the
    fp32 table ``cos_sin`` [max_position, D] (cos | sin); returns bf16 bits."""
    d = x_bits.shape[-1]
    half = d // 2
    cs = np.asarray(cos_sin, dtype=np.float32).reshape(-1, d)[np.asarray(positions, dtype=np.int64)]
    c = cs[:, None, :half]
    s = cs[:, None, half:]
    x = bf16_bits_to_f32(x_bits)
    x1, x2 = x[..., :half], x[..., half:]
    y1 = x1 * c - x2 * s
    y2 = x2 * c + x1 * s
    return f32_to_bf16_bits(np.concatenate([y1, y2], axis=-1))


def rope_store_kvcache(positions, q_bits, k_bits, v_bits, cos_sin, k_cache_bits, v_cache_bits, slot_mapping):
    """Roped query bits, and copies of the caches ([num_slots, Hk*D] uint16 views) with
    the roped key and the value rows stored at their slots (-1 skipped)."""
    q_out = rope_rows(q_bits, positions, cos_sin)
    k_rot = rope_rows(k_bits, positions, cos_sin)
    kc = np.array(k_cache_bits, copy=True)
    vc = np.array(v_cache_bits, copy=True)
    n = k_bits.shape[0]
    for i, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot == -1:
            continue
        kc[slot] = k_rot[i].reshape(-1)
        vc[slot] = np.asarray(v_bits)[i].reshape(-1)
    assert n == len(slot_mapping)
    return q_out, kc, vc
