"""ctypes binding of the C-ABI library ``libvlcache_b200.so``.

The library is the product: there is no Python or CPU fallback for any op.  If
the shared object is missing or fails to load, importing the ops raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libvlcache_b200.so"
_lib: ctypes.CDLL | None = None

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

# name -> (restype, argtypes); must match include/vlcache_b200.h
SIGNATURES: dict[str, tuple] = {
    "vlc_version": (c_int, []),
    "vlc_status_string": (ctypes.c_char_p, [c_int]),
    "vlc_get_device_error": (c_int, [c_int]),
    "vlc_selftest_bounded_wait": (c_int, [c_i64, c_int, c_vp]),
    "vlc_num_sms": (c_int, []),
    "vlc_store_kvcache": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_int, c_int, c_i64, c_vp]),
    "vlc_rope_store_kvcache": (c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                       c_int, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_int, c_int, c_int, c_int,
                                       c_vp]),
    "vlc_mrope_shift": (c_int, [c_vp, c_vp, c_i64, c_int, c_i64, c_int, c_int, c_vp, c_vp, c_int,
                                c_vp, c_vp, c_float, c_vp]),
    "vlc_prefill_plan": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_vp, c_i64, c_vp]),
    "vlc_prefill_plan_capacity": (c_i64, [c_vp, c_vp, c_int, c_int, c_int, c_int]),
    "vlc_attention_plan": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_int, c_vp, c_i64, c_vp]),
    "vlc_attention_plan_capacity": (c_i64, [c_vp, c_vp, c_int, c_int, c_int, c_int, c_int]),
    "vlc_prefill_workspace_size": (c_i64, [c_vp]),
    "vlc_prefill_set_kernel": (c_int, [c_int]),
    "vlc_prefill_attn": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_i64, c_i64, c_i64, c_int, c_int,
                                 c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "vlc_prefill_attn_inflight": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_i64, c_i64, c_i64, c_int, c_int,
                                          c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_i64, c_vp, c_i64,
                                          c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "vlc_decode_attn": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_i64, c_int, c_int, c_vp, c_int,
                                c_int, c_vp, c_int, c_float, c_vp, c_i64, c_vp, c_i64, c_vp]),
    "vlc_decode_workspace_size": (c_i64, [c_int, c_int, c_int, c_int]),
    "vlc_decode_attn_noalloc": (c_int, [c_vp, c_i64, c_int, c_int, c_vp, c_vp, c_i64, c_int, c_int, c_vp, c_int,
                                        c_int, c_vp, c_int, c_float, c_vp, c_i64, c_vp]),
    "vlc_decode_noalloc_scratch_bytes": (c_i64, []),
    "vlc_warm_metadata": (c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_vp, c_int, c_vp, c_vp,
                                  c_vp]),
    "vlc_content_hash_workspace_size": (c_i64, [c_i64]),
    "vlc_content_hash_device": (c_int, [c_vp, c_i64, c_vp, c_int, c_vp, c_i64, c_vp, c_vp]),
    "vlc_content_hash_host": (c_int, [c_vp, c_i64, c_vp, c_int, c_int, c_vp]),
    "vlc_xxh64": (ctypes.c_uint64, [c_vp, c_i64, ctypes.c_uint64]),
    "vlc_linear_workspace_size": (c_i64, [c_int, c_int, c_int, c_int]),
    "vlc_linear_set_kernel": (c_int, [c_int]),
    "vlc_linear": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_i64, c_int, c_int, c_int, c_vp, c_i64, c_vp]),
    "vlc_linear_silu_mul": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_int, c_int, c_int, c_vp, c_i64,
                                    c_vp]),
    "vlc_qkv_rope_store_kvcache": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp,
                                           c_vp, c_vp, c_i64, c_int, c_int, c_int, c_int, c_int, c_vp, c_i64,
                                           c_vp]),
}


class VLCError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, fn: str, status: int):
        self.status = status
        msg = lib().vlc_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"{fn} failed with status {status}: {msg}")


def lib_path() -> Path:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raises if it is not built."""
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(
                f"{_LIB_PATH} is missing: build it with `python -m vlcache_b200.build` "
                "(the CUDA kernels are required; there is no fallback path)")
        handle = ctypes.CDLL(str(_LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(fn_name: str, status: int) -> None:
    if status != 0:
        raise VLCError(fn_name, status)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
