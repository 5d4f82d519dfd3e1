"""The C-ABI library loads without a GPU and exports every entry point the header declares."""
import ctypes
import re
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent


def _declared_functions():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(vlc_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_exports_all_declared_symbols(cuda_lib):
    declared = _declared_functions()
    assert len(declared) >= 12
    raw = ctypes.CDLL(str(REPO / "vlcache_b200" / "libvlcache_b200.so"))
    for name in sorted(declared):
        assert hasattr(raw, name), name


def test_binding_table_matches_header(cuda_lib):
    from vlcache_b200._lib import exported_symbols
    assert set(exported_symbols()) == _declared_functions()


def test_status_strings_and_version(cuda_lib):
    assert cuda_lib.vlc_version() >= 100
    assert cuda_lib.vlc_status_string(0) == b"ok"
    assert b"workspace" in cuda_lib.vlc_status_string(6)


def test_argument_errors_are_reported_before_launch(cuda_lib):
    # NULL pointers / bad shapes return status codes without touching a device.
    one = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    assert cuda_lib.vlc_store_kvcache(None, 256, None, 256, None, None, None, 4, 256, 512, None) == 1
    assert cuda_lib.vlc_store_kvcache(one, 256, one, 256, one, one, one, 4, 250, 512, None) == 3
    sec = (ctypes.c_int32 * 3)(16, 24, 20)   # sums to 60 != 64
    d = (ctypes.c_int32 * 3)(1, 1, 1)
    assert cuda_lib.vlc_mrope_shift(one, None, 0, 1, 16, 2, 128, one, None, 1, d, sec, 1e6, None) == 2
    assert cuda_lib.vlc_decode_attn(one, 128, 1, 16, one, one, 256, 2, 64, one, 1, 256, one, 10, 1.0, one,
                                    128, None, 0, None) == 5
    # rotary + scatter: head_dim 64 unsupported (5), NULL query (1), fused mode without caches (1)
    assert cuda_lib.vlc_rope_store_kvcache(one, one, 512, one, 512, one, 128, one, 128, one, 64, 64, one, one, one,
                                           16, None, 0, 4, 4, 1, 64, None) == 5
    assert cuda_lib.vlc_rope_store_kvcache(one, None, 512, one, 512, one, 128, one, 128, one, 64, 128, one, one,
                                           one, 16, None, 0, 4, 4, 1, 128, None) == 1
    assert cuda_lib.vlc_rope_store_kvcache(one, one, 512, one, 512, one, 128, one, 128, one, 64, 128, None, None,
                                           one, 16, None, 0, 4, 4, 1, 128, None) == 1
    plan = np.zeros(32, np.int32)
    assert cuda_lib.vlc_prefill_attn(one, 2048, 1, 16, one, one, 256, 256, 256, 2, 128, one, 1, 256, one,
                                     plan.ctypes.data, 1.0, one, 2048, None, 0, None) == 8
