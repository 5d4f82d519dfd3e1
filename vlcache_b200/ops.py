"""Torch-facing wrappers over the C ABI (device pointers, strides, current stream).

These are thin: validate what the reference validates, hand raw pointers to the
library, raise on a non-zero status.  Every op runs its CUDA kernel; tensors on
the CPU are rejected (there is no CPU path in the product).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import check, lib

HEAD_DIM = 128
DEFAULT_MROPE_SECTION = (16, 24, 24)  # Qwen2.5-VL rope_scaling.mrope_section


_raw_device = getattr(torch._C, "_cuda_getDevice", None)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream() -> int:
    """Handle of the current device's current stream.  Read raw (no torch.cuda.Stream object,
    no device-availability probe): it is on every launch's host path."""
    if _raw_device is not None and _raw_stream is not None:
        return _raw_stream(_raw_device())
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int:
    """Device address of ``t`` (0 for None); every C-ABI argument is declared ``void*``."""
    return 0 if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("vlcache_b200 ops run on CUDA tensors only (no CPU fallback)")


def num_sms() -> int:
    return int(lib().vlc_num_sms())


def device_error(reset: bool = True) -> int:
    """Synchronise and return (and by default clear) the library's device error word."""
    return int(lib().vlc_get_device_error(1 if reset else 0))


# --------------------------------------------------------------------------- scatter
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """``k_cache.view(-1, D)[slot_mapping[i]] = key[i]`` (and V); slot -1 is skipped.

    Same contract and assertions as nanovllm/layers/attention.py:33-40.
    """
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    assert key.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16
    assert slot_mapping.dtype == torch.int32
    num_slots = k_cache.numel() // D
    st = lib().vlc_store_kvcache(_ptr(key), key.stride(0), _ptr(value), value.stride(0), _ptr(k_cache),
                                 _ptr(v_cache), _ptr(slot_mapping), N, D, num_slots, _stream())
    check("vlc_store_kvcache", st)


# --------------------------------------------------------------------------- rotary + scatter
def _rope_args(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor, cos_sin_cache: torch.Tensor):
    N, H, D = query.shape
    Hk = key.shape[1]
    assert key.shape[0] == N and key.shape[2] == D and positions.numel() == N
    assert query.stride(-1) == 1 and query.stride(1) == D and key.stride(-1) == 1 and key.stride(1) == D
    assert query.dtype == torch.bfloat16 and key.dtype == torch.bfloat16
    assert positions.dtype == torch.int64 and positions.is_contiguous()
    assert cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous()
    assert cos_sin_cache.shape[-1] == D and cos_sin_cache.numel() == cos_sin_cache.shape[0] * D
    return N, H, Hk, D, cos_sin_cache.shape[0]


def rotary_embedding(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor,
                     cos_sin_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate-half RoPE of ``query`` [N, H, D] and ``key`` [N, Hk, D] at ``positions``.

    Semantics of nanovllm/layers/rotary_embedding.py:37-48 (``cos_sin_cache[positions]``
    split into cos | sin, ``apply_rotary_emb`` :6-14 in fp32, result in bf16); returns new
    tensors like the reference.  ``cos_sin_cache`` is the reference's buffer
    ([max_position, 1, D] fp32) or the same values as [max_position, D].
    """
    _require_cuda(positions, query, key, cos_sin_cache)
    N, H, Hk, D, max_pos = _rope_args(positions, query, key, cos_sin_cache)
    q_out = torch.empty((N, H, D), dtype=query.dtype, device=query.device)
    k_out = torch.empty((N, Hk, D), dtype=key.dtype, device=key.device)
    st = lib().vlc_rope_store_kvcache(_ptr(positions), _ptr(query), query.stride(0), _ptr(q_out), q_out.stride(0),
                                      _ptr(key), key.stride(0), None, 0, _ptr(cos_sin_cache), max_pos, D, None,
                                      None, None, 0, _ptr(k_out), k_out.stride(0), N, H, Hk, D, _stream())
    check("vlc_rope_store_kvcache", st)
    return q_out, k_out


def rope_store_kvcache(positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                       cos_sin_cache: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       slot_mapping: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE of ``query`` and ``key`` fused with the paged KV scatter: returns the roped
    query (into ``out`` when given; ``out`` may be ``query``) and writes the roped key
    and the value rows to ``k_cache`` / ``v_cache`` row ``slot_mapping[i]`` (-1 skipped).

    One launch for what the reference does in two steps: ``rotary_emb(positions, q, k)``
    (rotary_embedding.py:37-48) and ``store_kvcache`` (attention.py:10-40, with its
    stride assertions :33-40).  The key's K rows reach the cache roped, bit-identical to
    roping then scattering.
    """
    _require_cuda(positions, query, key, value, cos_sin_cache, k_cache, v_cache, slot_mapping)
    N, H, Hk, D, max_pos = _rope_args(positions, query, key, cos_sin_cache)
    assert value.shape == key.shape and value.stride(-1) == 1 and value.stride(1) == D
    assert value.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16 and v_cache.dtype == torch.bfloat16
    row = Hk * D
    assert k_cache.stride(1) == row and v_cache.stride(1) == row    # as store_kvcache (attention.py:33-40)
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert slot_mapping.dtype == torch.int32 and slot_mapping.numel() == N and slot_mapping.is_contiguous()
    if out is None:
        out = torch.empty((N, H, D), dtype=query.dtype, device=query.device)
    assert out.shape == (N, H, D) and out.stride(-1) == 1 and out.stride(1) == D
    num_slots = k_cache.numel() // row
    st = lib().vlc_rope_store_kvcache(_ptr(positions), _ptr(query), query.stride(0), _ptr(out), out.stride(0),
                                      _ptr(key), key.stride(0), _ptr(value), value.stride(0), _ptr(cos_sin_cache),
                                      max_pos, D, _ptr(k_cache), _ptr(v_cache), _ptr(slot_mapping), num_slots,
                                      None, 0, N, H, Hk, D, _stream())
    check("vlc_rope_store_kvcache", st)
    return out


# --------------------------------------------------------------------------- M-RoPE shift
def mrope_shift(k_cache: torch.Tensor, v_cache: torch.Tensor | None, src_slots: torch.Tensor,
                dst_slots: torch.Tensor | None, delta_thw, mrope_section=DEFAULT_MROPE_SECTION,
                rope_theta: float = 1e6) -> None:
    """Re-rotate reused K rows of one layer by an M-RoPE position delta.

    ``k_cache``/``v_cache`` are one layer's ``[num_blocks, block_size, Hk, D]`` (or
    ``[num_slots, Hk, D]``) caches.  With ``dst_slots`` None the rotation is in place;
    otherwise K rows move (rotated) to ``dst_slots`` and V rows move verbatim.
    """
    _require_cuda(k_cache, v_cache, src_slots, dst_slots)
    assert k_cache.dtype == torch.bfloat16 and k_cache.is_contiguous()
    assert src_slots.dtype == torch.int32 and (dst_slots is None or dst_slots.dtype == torch.int32)
    Hk, hd = k_cache.shape[-2], k_cache.shape[-1]
    num_slots = k_cache.numel() // (Hk * hd)
    n = src_slots.numel()
    if dst_slots is not None:
        assert dst_slots.numel() == n
    d = (ctypes.c_int32 * 3)(*[int(x) for x in delta_thw])
    sec = (ctypes.c_int32 * 3)(*[int(x) for x in mrope_section])
    st = lib().vlc_mrope_shift(_ptr(k_cache), _ptr(v_cache), 0, 1, int(num_slots), int(Hk), int(hd),
                               _ptr(src_slots), _ptr(dst_slots), n, d, sec, float(rope_theta), _stream())
    check("vlc_mrope_shift", st)


def mrope_shift_all_layers(kv_cache: torch.Tensor, src_slots: torch.Tensor, dst_slots: torch.Tensor | None,
                           delta_thw, mrope_section=DEFAULT_MROPE_SECTION, rope_theta: float = 1e6) -> None:
    """Shift reused image rows of every layer of a ``[2, L, NB, BS, Hk, D]`` cache in one launch."""
    assert kv_cache.dim() == 6 and kv_cache.is_contiguous()
    L = kv_cache.shape[1]
    per_layer = kv_cache[0, 0].numel()
    k0 = kv_cache[0, 0]
    v0 = kv_cache[1, 0]
    Hk, hd = kv_cache.shape[4], kv_cache.shape[5]
    num_slots = kv_cache.shape[2] * kv_cache.shape[3]
    _require_cuda(kv_cache, src_slots, dst_slots)
    n = src_slots.numel()
    d = (ctypes.c_int32 * 3)(*[int(x) for x in delta_thw])
    sec = (ctypes.c_int32 * 3)(*[int(x) for x in mrope_section])
    st = lib().vlc_mrope_shift(_ptr(k0), _ptr(v0) if dst_slots is not None else ctypes.c_void_p(0),
                               per_layer, L, num_slots, Hk, hd, _ptr(src_slots), _ptr(dst_slots), n, d, sec,
                               float(rope_theta), _stream())
    check("vlc_mrope_shift", st)


# --------------------------------------------------------------------------- prefill
@dataclass
class PrefillPlan:
    """Host plan (numpy int32) plus its device copy and workspace size (bytes)."""
    host: np.ndarray
    dev: torch.Tensor | None
    workspace_bytes: int

    @property
    def host_ptr(self) -> int:
        """Address of ``host`` (cached: the launch path passes it on every call)."""
        p = self.__dict__.get("_host_ptr")
        if p is None:
            p = self.__dict__["_host_ptr"] = int(self.host.ctypes.data)
        return p

    @property
    def grid(self) -> int:
        return int(self.host[2])

    @property
    def num_units(self) -> int:
        return int(self.host[3])

    @property
    def num_parts(self) -> int:
        return int(self.host[4])

    @property
    def num_merges(self) -> int:
        return int(self.host[5])

    def split_tiles(self) -> list[tuple[int, int, int]]:
        """(first query row, query rows, KV head) of every tile whose keys are split over
        several units (its output goes through the log-sum-exp merge of partials)."""
        off, n = int(self.host[14]), self.num_merges
        rec = self.host[off:off + 8 * n].reshape(n, 8) if n else np.zeros((0, 8), np.int32)
        return [(int(r[0]), int(r[1]), int(r[2])) for r in rec]


PREFILL_DEFAULT, PREFILL_PAIRS, PREFILL_QUADS = 0, 1, 2


def set_prefill_kernel(mode: int) -> None:
    """Unit kind of the prefill plans built from now on: ``PREFILL_PAIRS`` (two query tiles
    per unit on one SM), ``PREFILL_QUADS`` (four tiles per unit on a CTA pair) or
    ``PREFILL_DEFAULT``.  Each plan records its kind; the launch follows the plan."""
    check("vlc_prefill_set_kernel", lib().vlc_prefill_set_kernel(int(mode)))


def build_prefill_plan(cu_seqlens_q, cu_seqlens_k, num_heads: int, num_kv_heads: int, head_dim: int = HEAD_DIM,
                       num_sms: int = 0, device: torch.device | str | None = None, causal: bool = True) -> PrefillPlan:
    """Plan the warm-prefill attention launch from HOST cu_seqlens (lists/arrays/CPU tensors).
    ``causal=False`` plans the non-causal varlen attention (every row sees all keys of its
    sequence); ``head_dim`` may be 80..128 in steps of 16."""
    cq = np.ascontiguousarray(np.asarray(cu_seqlens_q, dtype=np.int32))
    ck = np.ascontiguousarray(np.asarray(cu_seqlens_k, dtype=np.int32))
    nseq = len(cq) - 1
    assert len(ck) == nseq + 1
    L = lib()
    sms = int(num_sms) if num_sms else (L.vlc_num_sms() if device is not None else 148)
    cap = L.vlc_attention_plan_capacity(cq.ctypes.data, ck.ctypes.data, nseq, num_heads, num_kv_heads,
                                        1 if causal else 0, sms)
    if cap < 0:
        raise ValueError("invalid prefill metadata (cu_seqlens / heads)")
    plan = np.zeros(int(cap), dtype=np.int32)
    used = ctypes.c_int64(0)
    st = L.vlc_attention_plan(cq.ctypes.data, ck.ctypes.data, nseq, num_heads, num_kv_heads, head_dim,
                              1 if causal else 0, sms, plan.ctypes.data, int(cap), ctypes.byref(used))
    check("vlc_attention_plan", st)
    plan = plan[: used.value].copy()
    ws = int(L.vlc_prefill_workspace_size(plan.ctypes.data))
    dev = None
    if device is not None:
        dev = torch.from_numpy(plan).pin_memory().to(device, non_blocking=True)
    return PrefillPlan(host=plan, dev=dev, workspace_bytes=ws)


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_tables: torch.Tensor | None,
                      plan: PrefillPlan, softmax_scale: float, out: torch.Tensor | None = None,
                      workspace: torch.Tensor | None = None, k_new: torch.Tensor | None = None,
                      v_new: torch.Tensor | None = None) -> torch.Tensor:
    """Causal (bottom-right) varlen attention — the flash_attn_varlen_func contract.

    Paged: ``k``/``v`` are one layer's ``[num_blocks, block_size, Hk, D]`` caches and
    ``block_tables`` maps sequences to pages.  Contiguous (``block_tables`` None): ``k``/``v``
    are ``[total_k, Hk, D]`` (any token stride) laid out by cu_seqlens_k.
    The kernel is a programmatic dependent launch of the previous kernel on the
    stream: that kernel may produce q/k/v, but not the plan or ``block_tables``.

    Paged with ``k_new``/``v_new`` (the step's in-flight ``[total_q, Hk, D]`` rows, row i
    for query row i): sequences with q_len == k_len read their keys from those rows and
    start without waiting for the previous kernel, which may then only write the cache
    (the KV scatter, an ordinary launch) — ``vlc_prefill_attn_inflight``.
    """
    _require_cuda(q, k, v, block_tables)
    assert q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
    total_q, H, hd = q.shape
    assert q.stride(2) == 1 and q.stride(1) == hd
    Hk = k.shape[-2]
    assert k.stride(-1) == 1 and k.stride(-2) == hd and v.stride(-1) == 1 and v.stride(-2) == hd
    if block_tables is not None:
        assert k.dim() == 4 and k.is_contiguous() and v.is_contiguous()
        block_size = k.shape[1]
        rows = k.shape[0] * k.shape[1]
        k_stride = v_stride = Hk * hd
        assert block_tables.dtype == torch.int32 and block_tables.stride(-1) == 1
        bt_ptr, bt_stride = _ptr(block_tables), block_tables.stride(0)
    else:
        assert k.dim() == 3 and v.dim() == 3 and k.shape[0] == v.shape[0]
        block_size, rows = 0, k.shape[0]
        k_stride, v_stride = k.stride(0), v.stride(0)
        bt_ptr, bt_stride = ctypes.c_void_p(0), 0
    if out is None:
        out = torch.empty(total_q, H, hd, dtype=q.dtype, device=q.device)
    assert out.stride(2) == 1 and out.stride(1) == hd
    if plan.dev is None or plan.dev.device != q.device:
        plan.dev = torch.from_numpy(plan.host).to(q.device)
    if plan.workspace_bytes > 0 and (workspace is None or workspace.numel() * workspace.element_size()
                                     < plan.workspace_bytes):
        workspace = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if k_new is not None:
        assert block_tables is not None and v_new is not None, "in-flight K/V go with a paged cache"
        _require_cuda(k_new, v_new)
        assert k_new.dim() == 3 and v_new.dim() == 3 and k_new.shape[1:] == (Hk, hd) and v_new.shape[1:] == (Hk, hd)
        assert k_new.shape[0] == v_new.shape[0] >= total_q
        assert k_new.stride(-1) == 1 and k_new.stride(-2) == hd and v_new.stride(-1) == 1 and v_new.stride(-2) == hd
        st = lib().vlc_prefill_attn_inflight(_ptr(q), q.stride(0), total_q, H, _ptr(k), _ptr(v), k_stride, v_stride,
                                             rows, Hk, hd, bt_ptr, bt_stride, block_size, _ptr(plan.dev),
                                             plan.host_ptr, float(softmax_scale), _ptr(out), out.stride(0),
                                             _ptr(workspace), ws_bytes, _ptr(k_new), _ptr(v_new), k_new.stride(0),
                                             v_new.stride(0), k_new.shape[0], _stream())
        check("vlc_prefill_attn_inflight", st)
        return out
    st = lib().vlc_prefill_attn(_ptr(q), q.stride(0), total_q, H, _ptr(k), _ptr(v), k_stride, v_stride, rows,
                                Hk, hd, bt_ptr, bt_stride, block_size, _ptr(plan.dev), plan.host_ptr,
                                float(softmax_scale), _ptr(out), out.stride(0), _ptr(workspace), ws_bytes,
                                _stream())
    check("vlc_prefill_attn", st)
    return out


# --------------------------------------------------------------------------- decode
def decode_workspace_bytes(num_seqs: int, num_heads: int, num_kv_heads: int, max_context_len: int) -> int:
    return int(lib().vlc_decode_workspace_size(num_seqs, num_heads, num_kv_heads, max_context_len))


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                     context_lens: torch.Tensor, max_context_len: int, softmax_scale: float,
                     out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One-token paged decode (flash_attn_with_kvcache contract); q/out are ``[B, H, D]``."""
    _require_cuda(q, k_cache, v_cache, block_tables, context_lens)
    if q.dim() == 4:
        q = q.squeeze(1)
    B, H, hd = q.shape
    assert q.stride(2) == 1 and q.stride(1) == hd
    Hk = k_cache.shape[-2]
    block_size = k_cache.shape[1] if k_cache.dim() == 4 else 256
    num_slots = k_cache.numel() // (Hk * hd)
    assert context_lens.dtype == torch.int32 and block_tables.dtype == torch.int32
    if out is None:
        out = torch.empty(B, H, hd, dtype=q.dtype, device=q.device)
    need = decode_workspace_bytes(B, H, Hk, max_context_len)
    if need > 0 and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = lib().vlc_decode_attn(_ptr(q), q.stride(0), B, H, _ptr(k_cache), _ptr(v_cache), num_slots, Hk, hd,
                               _ptr(block_tables), block_tables.stride(0), block_size, _ptr(context_lens),
                               int(max_context_len), float(softmax_scale), _ptr(out), out.stride(0),
                               _ptr(workspace), ws_bytes, _stream())
    check("vlc_decode_attn", st)
    return out


# --------------------------------------------------------------------------- metadata
VSEQ_INTS, REUSE_INTS = 7, 8


def warm_metadata(desc: torch.Tensor, num_vseqs: int, reuse_offset: int, num_reuse: int, table_offset: int,
                  block_size: int, total_q: int, total_slots: int, table_rows: int, table_width: int,
                  total_reuse: int):
    """Device warm-prefill metadata from one int32 descriptor buffer ``desc`` =
    [virtual-sequence descriptors][reuse descriptors at reuse_offset][flat block tables at
    table_offset] (layout in include/vlcache_b200.h, vlc_warm_metadata).  Returns
    (positions int64, slot_mapping int32, block_tables int32 or None, src_slots, dst_slots)."""
    _require_cuda(desc)
    assert desc.dtype == torch.int32 and desc.is_contiguous()
    dev = desc.device
    positions = torch.empty(total_q, dtype=torch.int64, device=dev)
    slots = torch.empty(total_slots, dtype=torch.int32, device=dev)
    tables = torch.empty(table_rows, table_width, dtype=torch.int32, device=dev) if table_rows > 0 else None
    src = torch.empty(total_reuse, dtype=torch.int32, device=dev)
    dst = torch.empty(total_reuse, dtype=torch.int32, device=dev)
    base = desc.data_ptr()
    st = lib().vlc_warm_metadata(ctypes.c_void_p(base), num_vseqs, ctypes.c_void_p(base + 4 * reuse_offset),
                                 num_reuse, ctypes.c_void_p(base + 4 * table_offset), block_size,
                                 _ptr(positions), _ptr(slots) if total_slots > 0 else ctypes.c_void_p(0),
                                 _ptr(tables), table_width if tables is not None else 0, _ptr(src), _ptr(dst),
                                 _stream())
    check("vlc_warm_metadata", st)
    return positions, slots, tables, src, dst


# --------------------------------------------------------------------------- linear layers
LINEAR, SILU_MUL, QKV_ROPE = 0, 1, 2
_LINEAR_WS: dict = {}


def linear_workspace(kind: int, m: int, n: int, k: int, device) -> tuple[torch.Tensor | None, int]:
    """The stream-K workspace of a linear launch: one zeroed buffer per device, grown to
    the largest size asked for (each launch leaves it zeroed; launches on one stream never
    overlap).  Returns (tensor, bytes)."""
    need = int(lib().vlc_linear_workspace_size(kind, m, n, k))
    if need <= 0:
        return None, 0
    dev = torch.device(device)
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    ws = _LINEAR_WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        _LINEAR_WS[key] = ws
    return ws, ws.numel()


def set_linear_kernel(mode: int) -> None:
    """GEMM kernel of the linear ops, process-wide: 0 automatic (a cost model picks per
    shape), 1 single-SM 128 x 256 tiles (stream-K where it pays), 2 CTA pairs
    (tcgen05.mma.cta_group::2, 256 x 256), 3 single-SM 128 x 128, 4 single-SM 128 x 224
    (plain linear only; the fused epilogues fall back to pairs)."""
    check("vlc_linear_set_kernel", lib().vlc_linear_set_kernel(int(mode)))


def reset_linear_workspaces() -> None:
    """Zero the cached stream-K workspaces (after a recorded device error)."""
    for ws in _LINEAR_WS.values():
        ws.zero_()


def _linear_args(x: torch.Tensor, weight: torch.Tensor):
    _require_cuda(x, weight)
    assert x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1]
    assert x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
    assert x.stride(1) == 1 and weight.stride(1) == 1
    return x.shape[0], x.shape[1]


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None, stream_k: bool = True) -> torch.Tensor:
    """``F.linear(x, weight, bias)`` for bf16 ``x`` [m, k] and ``weight`` [n, k] on the
    tcgen05 GEMM (nanovllm/layers/linear.py:73, :154); ``stream_k=False`` runs whole
    output tiles per CTA (no workspace)."""
    m, k = _linear_args(x, weight)
    n = weight.shape[0]
    if bias is not None:
        _require_cuda(bias)
        assert bias.dtype == torch.bfloat16 and bias.is_contiguous() and bias.numel() == n
    if out is None:
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    assert out.shape == (m, n) and out.stride(1) == 1
    ws, ws_bytes = linear_workspace(LINEAR, m, n, k, x.device) if stream_k else (None, 0)
    st = lib().vlc_linear(_ptr(x), x.stride(0), _ptr(weight), weight.stride(0), _ptr(bias), _ptr(out),
                          out.stride(0), m, n, k, _ptr(ws), ws_bytes, _stream())
    check("vlc_linear", st)
    return out


def linear_silu_mul(x: torch.Tensor, gate_up_weight: torch.Tensor, out: torch.Tensor | None = None,
                    stream_k: bool = True) -> torch.Tensor:
    """``SiluAndMul()(F.linear(x, gate_up_weight))`` in one kernel: ``gate_up_weight`` is
    [2 I, k] (gate rows then up rows); returns silu(gate) * up, [m, I]
    (nanovllm/models/qwen3.py:112-114, nanovllm/layers/activation.py:8-14)."""
    m, k = _linear_args(x, gate_up_weight)
    assert gate_up_weight.shape[0] % 2 == 0
    inter = gate_up_weight.shape[0] // 2
    if out is None:
        out = torch.empty(m, inter, dtype=x.dtype, device=x.device)
    assert out.shape == (m, inter) and out.stride(1) == 1
    ws, ws_bytes = linear_workspace(SILU_MUL, m, inter, k, x.device) if stream_k else (None, 0)
    st = lib().vlc_linear_silu_mul(_ptr(x), x.stride(0), _ptr(gate_up_weight), gate_up_weight.stride(0), _ptr(out),
                                   out.stride(0), m, inter, k, _ptr(ws), ws_bytes, _stream())
    check("vlc_linear_silu_mul", st)
    return out


def qkv_rope_store_kvcache(x: torch.Tensor, qkv_weight: torch.Tensor, qkv_bias: torch.Tensor | None,
                           positions: torch.Tensor, cos_sin_cache: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, slot_mapping: torch.Tensor, num_heads: int, num_kv_heads: int,
                           q_out: torch.Tensor | None = None, stream_k: bool = True) -> torch.Tensor:
    """The QKV projection of the recomputed rows, its bias, the rotary embedding and the
    KV scatter in one kernel; returns the roped q [m, num_heads, 128] and writes the
    roped k and the v rows to the paged cache at ``slot_mapping`` (-1 skipped).
    Same result as ``qkv = F.linear(x, W, b)``; split; ``rotary_emb(positions, q, k)``;
    ``store_kvcache(k, v, ...)`` (nanovllm/models/qwen3.py:75-84), up to the GEMM's
    accumulation order."""
    m, hidden = _linear_args(x, qkv_weight)
    D = HEAD_DIM
    assert qkv_weight.shape[0] == (num_heads + 2 * num_kv_heads) * D
    _require_cuda(qkv_bias, positions, cos_sin_cache, k_cache, v_cache, slot_mapping)
    if qkv_bias is not None:
        assert qkv_bias.dtype == torch.bfloat16 and qkv_bias.is_contiguous()
    assert positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == m
    assert cos_sin_cache.dtype == torch.float32 and cos_sin_cache.is_contiguous()
    assert cos_sin_cache.shape[-1] == D and cos_sin_cache.numel() == cos_sin_cache.shape[0] * D
    row = num_kv_heads * D
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert tuple(k_cache.shape[-2:]) == (num_kv_heads, D) and tuple(v_cache.shape) == tuple(k_cache.shape)
    assert slot_mapping.dtype == torch.int32 and slot_mapping.numel() == m and slot_mapping.is_contiguous()
    if q_out is None:
        q_out = torch.empty(m, num_heads, D, dtype=x.dtype, device=x.device)
    assert q_out.shape == (m, num_heads, D) and q_out.stride(2) == 1 and q_out.stride(1) == D
    ws, ws_bytes = linear_workspace(QKV_ROPE, m, qkv_weight.shape[0], hidden, x.device) if stream_k else (None, 0)
    st = lib().vlc_qkv_rope_store_kvcache(_ptr(x), x.stride(0), _ptr(qkv_weight), qkv_weight.stride(0),
                                          _ptr(qkv_bias), _ptr(positions), _ptr(cos_sin_cache),
                                          cos_sin_cache.shape[0], _ptr(q_out), q_out.stride(0), _ptr(k_cache),
                                          _ptr(v_cache), _ptr(slot_mapping), k_cache.numel() // row, m, hidden,
                                          num_heads, num_kv_heads, D, _ptr(ws), ws_bytes, _stream())
    check("vlc_qkv_rope_store_kvcache", st)
    return q_out


# --------------------------------------------------------------------------- content hash
def _header_buf(header: bytes):
    hb = bytes(header)
    return ctypes.create_string_buffer(hb, max(1, len(hb))), len(hb)


def content_hash_device_async(data: torch.Tensor, header: bytes = b"",
                              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Tree-XXH64 digest (include/vlcache_b200.h, vlc_content_hash_*) of a CUDA tensor's
    bytes with ``header``, as a one-element int64 device tensor (the uint64 bit pattern),
    computed on the current stream without any host synchronisation."""
    _require_cuda(data)
    assert data.is_contiguous(), "hash a contiguous tensor"
    nbytes = data.numel() * data.element_size()
    need = int(lib().vlc_content_hash_workspace_size(nbytes))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=data.device)
    out = torch.empty(1, dtype=torch.int64, device=data.device)
    hb, hl = _header_buf(header)
    st = lib().vlc_content_hash_device(_ptr(data), nbytes, hb, hl, _ptr(workspace),
                                       workspace.numel() * workspace.element_size(), _ptr(out), _stream())
    check("vlc_content_hash_device", st)
    return out


def content_hash(data: torch.Tensor | np.ndarray, header: bytes = b"", num_threads: int = 0) -> int:
    """Tree-XXH64 digest of a tensor's bytes as a Python int: on the GPU when the tensor
    lives there (one 8-byte read back), else on the host threads."""
    if torch.is_tensor(data) and data.is_cuda:
        return int(content_hash_device_async(data, header).item()) & (2 ** 64 - 1)
    arr = np.ascontiguousarray(data.numpy() if torch.is_tensor(data) else data)
    hb, hl = _header_buf(header)
    out = ctypes.c_uint64(0)
    st = lib().vlc_content_hash_host(ctypes.c_void_p(arr.ctypes.data), arr.nbytes, hb, hl, num_threads,
                                     ctypes.byref(out))
    check("vlc_content_hash_host", st)
    return int(out.value)


def xxh64(data: bytes | np.ndarray, seed: int = 0) -> int:
    """Plain XXH64 of host bytes (the tree's primitive)."""
    arr = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    return int(lib().vlc_xxh64(ctypes.c_void_p(arr.ctypes.data if arr.size else 0), arr.size, seed))
