"""Seeded synthetic workloads shared by the tests and the bench (shapes from BASELINE configs)."""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

QWEN_3B = dict(num_heads=16, num_kv_heads=2, num_layers=36)
QWEN_7B = dict(num_heads=28, num_kv_heads=4, num_layers=28)
HEAD_DIM = 128


@dataclass
class WarmCase:
    """One warm-prefill attention problem in nano-vllm's varlen/paged layout."""
    q: torch.Tensor              # [total_q, H, D]
    k_cache: torch.Tensor        # [NB, BS, Hk, D]
    v_cache: torch.Tensor
    block_tables: torch.Tensor   # [num_virtual_seqs, width] int32 (-1 padded)
    cu_q: np.ndarray
    cu_k: np.ndarray
    scale: float


def warm_request_meta(prefix: int, n_img: int, suffix: int, R: int, first_block: int = 0, block_size: int = 256):
    """cu_seqlens / block table of one warm request (two virtual sub-sequences,
    nanovllm/engine/model_runner.py:232-276)."""
    n = prefix + n_img + suffix
    img_start, img_end = prefix, prefix + n_img
    nb = (n + block_size - 1) // block_size
    bt = list(range(first_block, first_block + nb))
    a = img_start + R
    cu_q = [0, a, a + (n - img_end)]
    cu_k = [0, a, a + n]
    return n, bt, cu_q, cu_k


def make_warm_case(specs, num_heads, num_kv_heads, dtype=torch.bfloat16, device="cpu", seed=0,
                   block_size=256, shuffle_blocks=True, extra_blocks=3) -> WarmCase:
    """specs: list of (prefix, n_img, suffix, R).  Each warm request gets its own pages
    (shuffled block ids to exercise the block table)."""
    g = torch.Generator().manual_seed(seed)
    metas = []
    nb_total = 0
    for (pre, ni, suf, R) in specs:
        n, bt, cq, ck = warm_request_meta(pre, ni, suf, R, nb_total, block_size)
        metas.append((n, bt, cq, ck))
        nb_total += len(bt)
    nb_total += extra_blocks
    perm = torch.randperm(nb_total, generator=g).tolist() if shuffle_blocks else list(range(nb_total))
    cu_q, cu_k, bts = [0], [0], []
    for (n, bt, cq, ck) in metas:
        bt = [perm[b] for b in bt]
        for i in range(2):
            cu_q.append(cu_q[-1] + (cq[i + 1] - cq[i]))
            cu_k.append(cu_k[-1] + (ck[i + 1] - ck[i]))
            bts.append(bt)
    width = max(len(b) for b in bts)
    block_tables = torch.tensor([b + [-1] * (width - len(b)) for b in bts], dtype=torch.int32)
    total_q = cu_q[-1]
    q = torch.randn(total_q, num_heads, HEAD_DIM, generator=g).to(dtype)
    k_cache = torch.randn(nb_total, block_size, num_kv_heads, HEAD_DIM, generator=g).to(dtype)
    v_cache = torch.randn(nb_total, block_size, num_kv_heads, HEAD_DIM, generator=g).to(dtype)
    return WarmCase(q.to(device), k_cache.to(device), v_cache.to(device), block_tables.to(device),
                    np.asarray(cu_q, np.int32), np.asarray(cu_k, np.int32), 1.0 / math.sqrt(HEAD_DIM))


def cfg2_spec(ratio=0.1):
    """Qwen2.5-VL-3B, 3840x2160 image: 77x137 = 10,549 vision tokens, 20 + 48 text tokens."""
    n_img = 77 * 137
    return [(20, n_img, 48, int(math.ceil(ratio * n_img)))]


def make_decode_case(num_seqs, num_heads, num_kv_heads, lens, dtype=torch.bfloat16, device="cpu", seed=0,
                     block_size=256):
    g = torch.Generator().manual_seed(seed)
    lens = [int(x) for x in lens]
    nbs = [(n + block_size - 1) // block_size for n in lens]
    total = sum(nbs) + 2
    perm = torch.randperm(total, generator=g).tolist()
    bts, pos = [], 0
    for nb in nbs:
        bts.append(perm[pos:pos + nb])
        pos += nb
    width = max(nbs)
    block_tables = torch.tensor([b + [-1] * (width - len(b)) for b in bts], dtype=torch.int32)
    q = torch.randn(num_seqs, num_heads, HEAD_DIM, generator=g).to(dtype)
    k_cache = torch.randn(total, block_size, num_kv_heads, HEAD_DIM, generator=g).to(dtype)
    v_cache = torch.randn(total, block_size, num_kv_heads, HEAD_DIM, generator=g).to(dtype)
    ctx = torch.tensor(lens, dtype=torch.int32)
    return (q.to(device), k_cache.to(device), v_cache.to(device), block_tables.to(device), ctx.to(device),
            1.0 / math.sqrt(HEAD_DIM))


def poison_unused_slots(cache: torch.Tensor, block_tables, lens_per_row) -> None:
    """Fill cache slots past each sequence's length (inside its last page) with NaN,
    the way never-written cache memory may look."""
    bs = cache.shape[1]
    bt = np.asarray(block_tables.cpu() if torch.is_tensor(block_tables) else block_tables)
    for row, n in enumerate(lens_per_row):
        nb = (n + bs - 1) // bs
        if n % bs:
            cache[int(bt[row][nb - 1]), n % bs:] = float("nan")


def attn_errors(out: torch.Tensor, ref: torch.Tensor):
    d = (out.float().cpu() - ref.float().cpu()).abs()
    return float(d.max()), float(d.mean())


@dataclass
class Cfg1Case(WarmCase):
    k_cache_old: torch.Tensor = None   # vision K rotated at the old offset 0 (what the cache holds)
    vision_slots: torch.Tensor = None  # slots of the 1,024 vision rows


def make_cfg1_case(dtype=torch.float32, device="cpu") -> Cfg1Case:
    """Qwen2.5-VL-3B attention shapes, seed 0, 16 prefix text tokens,
    1,024 vision tokens (32x32 merged grid), 32 suffix text tokens.  Cached vision K is
    rotated (M-RoPE [16,24,24], theta 1e6) at vision start 0; the warm request places the
    image at start 16.  Queries: the 16 prefix rows, the first 102 vision rows and the 32
    suffix rows (150), causal by logical position over 1,072 keys, scale 1/sqrt(128).
    ``k_cache`` holds K rotated at the NEW positions (the fp32 truth); ``k_cache_old``
    holds the cached rows at the old positions (input of the position-shift kernel)."""
    from oracle import mrope as omr
    H, Hk, D = 16, 2, 128
    pre, n_img, suf, R = 16, 1024, 32, 102
    n = pre + n_img + suf
    g = torch.Generator().manual_seed(0)
    k_pre = torch.randn(pre, Hk, D, generator=g)
    k_raw = torch.randn(n_img, Hk, D, generator=g)
    k_suf = torch.randn(suf, Hk, D, generator=g)
    v = torch.randn(n, Hk, D, generator=g)
    q = torch.randn(pre + R + suf, H, D, generator=g)
    k_old = omr.apply_mrope(k_raw, omr.vision_positions(0, 32, 32))
    k_new = omr.apply_mrope(k_raw, omr.vision_positions(pre, 32, 32))
    nb = 8
    perm = torch.randperm(nb, generator=g).tolist()
    bt = perm[:(n + 255) // 256]
    kc_new = torch.zeros(nb, 256, Hk, D)
    kc_old = torch.zeros(nb, 256, Hk, D)
    vc = torch.zeros(nb, 256, Hk, D)
    slots = torch.tensor([bt[p // 256] * 256 + p % 256 for p in range(n)], dtype=torch.long)
    full_new = torch.cat([k_pre, k_new, k_suf])
    full_old = torch.cat([k_pre, k_old, k_suf])
    kc_new.view(-1, Hk, D)[slots] = full_new
    kc_old.view(-1, Hk, D)[slots] = full_old
    vc.view(-1, Hk, D)[slots] = v
    cu_q = np.asarray([0, pre + R, pre + R + suf], np.int32)
    cu_k = np.asarray([0, pre + R, pre + R + n], np.int32)
    block_tables = torch.tensor([bt, bt], dtype=torch.int32)
    return Cfg1Case(q.to(dtype).to(device), kc_new.to(dtype).to(device), vc.to(dtype).to(device),
                    block_tables.to(device), cu_q, cu_k, 1.0 / math.sqrt(D),
                    k_cache_old=kc_old.to(dtype).to(device),
                    vision_slots=slots[pre:pre + n_img].to(torch.int32).to(device))
