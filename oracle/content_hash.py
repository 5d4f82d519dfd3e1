"""CPU restatement of the encoder-cache content hash (test oracle only).

Only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s reference leg use this
module, as the checker; the product path never calls it.

* ``xxh64`` restates XXH64 from the xxHash specification (xxhash 3.x, the hash the
  reference calls in nanovllm/engine/encoder_cache_manager.py:24-29): 4 accumulators
  over 32-byte stripes, round ``rotl(acc + in * P2, 31) * P1``, merge, tail, avalanche.
  ``tests/golden/xxh64_vectors.npz`` (made by ``tests/golden/make_hash_golden.py`` with
  the ``xxhash`` package) pins it.
* ``tree_hash`` is the library's parallel content hash built from that primitive
  (include/vlcache_b200.h, vlc_content_hash_*): level 1 XXH64 (seed 1) of 1 KB chunks,
  level 2 XXH64 (seed 2) of the level-1 digests in 512-byte chunks (64 digests), level 3
  XXH64 (seed 3) of the level-2 digests in 1 KB chunks, then XXH64 (seed 4) of the
  little-endian words {header_len, header zero-padded to 8 bytes, nbytes, n1, d3...}.
numpy uint64 arithmetic wraps like the C code; level 1 is vectorised over chunks.
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1
P1, P2, P3, P4, P5 = (0x9E3779B185EBCA87, 0xC2B2AE3D27D4EB4F, 0x165667B19E3779F9, 0x85EBCA77C2B2AE63,
                      0x27D4EB2F165667C5)
CHUNK = 1024


def _rotl(x: int, r: int) -> int:
    return ((x << r) | (x >> (64 - r))) & M64


def _round(acc: int, inp: int) -> int:
    return (_rotl((acc + inp * P2) & M64, 31) * P1) & M64


def _merge(acc: int, v: int) -> int:
    return ((acc ^ _round(0, v)) * P1 + P4) & M64


def _avalanche(h: int) -> int:
    h ^= h >> 33
    h = (h * P2) & M64
    h ^= h >> 29
    h = (h * P3) & M64
    return h ^ (h >> 32)


def xxh64(data: bytes, seed: int = 0) -> int:
    """XXH64 of ``data`` (bytes) with ``seed``."""
    b = bytes(data)
    n = len(b)
    seed &= M64
    i = 0
    if n >= 32:
        v = [(seed + P1 + P2) & M64, (seed + P2) & M64, seed, (seed - P1) & M64]
        while i + 32 <= n:
            for k in range(4):
                v[k] = _round(v[k], int.from_bytes(b[i + 8 * k:i + 8 * k + 8], "little"))
            i += 32
        h = (_rotl(v[0], 1) + _rotl(v[1], 7) + _rotl(v[2], 12) + _rotl(v[3], 18)) & M64
        for k in range(4):
            h = _merge(h, v[k])
    else:
        h = (seed + P5) & M64
    h = (h + n) & M64
    while i + 8 <= n:
        h ^= _round(0, int.from_bytes(b[i:i + 8], "little"))
        h = (_rotl(h, 27) * P1 + P4) & M64
        i += 8
    if i + 4 <= n:
        h ^= (int.from_bytes(b[i:i + 4], "little") * P1) & M64
        h = (_rotl(h, 23) * P2 + P3) & M64
        i += 4
    while i < n:
        h ^= (b[i] * P5) & M64
        h = (_rotl(h, 11) * P1) & M64
        i += 1
    return _avalanche(h)


def _np_rotl(x, r):
    return (x << np.uint64(r)) | (x >> np.uint64(64 - r))


def _np_round(acc, inp):
    with np.errstate(over="ignore"):
        return _np_rotl(acc + inp * np.uint64(P2), 31) * np.uint64(P1)


def _xxh64_full_chunks(words: np.ndarray, seed: int) -> np.ndarray:
    """XXH64 of each row of ``words`` [n, chunk // 8] (full chunks of a multiple of 32
    bytes), vectorised."""
    n, nw = words.shape
    with np.errstate(over="ignore"):
        v = [np.full(n, (seed + P1 + P2) & M64, np.uint64), np.full(n, (seed + P2) & M64, np.uint64),
             np.full(n, seed & M64, np.uint64), np.full(n, (seed - P1) & M64, np.uint64)]
        for s in range(nw // 4):
            for k in range(4):
                v[k] = _np_round(v[k], words[:, 4 * s + k])
        h = _np_rotl(v[0], 1) + _np_rotl(v[1], 7) + _np_rotl(v[2], 12) + _np_rotl(v[3], 18)
        for k in range(4):
            h = (h ^ _np_round(np.zeros(n, np.uint64), v[k])) * np.uint64(P1) + np.uint64(P4)
        h = h + np.uint64(8 * nw)
        h ^= h >> np.uint64(33)
        h = h * np.uint64(P2)
        h ^= h >> np.uint64(29)
        h = h * np.uint64(P3)
        h ^= h >> np.uint64(32)
    return h


def _level(buf: np.ndarray, seed: int, chunk: int = CHUNK) -> np.ndarray:
    """XXH64 (``seed``) of every ``chunk``-byte piece of ``buf`` (the last one shorter)."""
    n = buf.size
    full = n // chunk
    out = np.zeros((n + chunk - 1) // chunk, np.uint64)
    if full:
        out[:full] = _xxh64_full_chunks(buf[:full * chunk].view("<u8").reshape(full, chunk // 8), seed)
    if n % chunk:
        out[full] = xxh64(buf[full * chunk:].tobytes(), seed)
    return out


def tree_hash(data: bytes | np.ndarray, header: bytes = b"") -> int:
    """The library's content hash of ``data`` with ``header`` (at most 256 bytes)."""
    buf = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data).reshape(-1).view(np.uint8)
    d1 = _level(buf, 1)
    d2 = _level(d1.astype("<u8").view(np.uint8), 2, 512) if d1.size else np.zeros(0, np.uint64)
    d3 = _level(d2.astype("<u8").view(np.uint8), 3) if d2.size else np.zeros(0, np.uint64)
    hb = bytes(header)
    hw = (len(hb) + 7) // 8
    padded = np.frombuffer(hb + b"\0" * (8 * hw - len(hb)), "<u8") if hw else np.zeros(0, "<u8")
    words = np.concatenate([np.array([len(hb)], "<u8"), padded, np.array([buf.size, d1.size], "<u8"),
                            d3.astype("<u8")])
    return xxh64(words.tobytes(), 4)
