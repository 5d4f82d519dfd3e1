"""Encoder-cache content hash on the host (no GPU): the XXH64 primitive of the oracle and
of the library against digests the ``xxhash`` package produced (the hash the reference
calls, nanovllm/engine/encoder_cache_manager.py:24-29), the library's host tree hash
against the oracle's, and the cache manager's LRU policy against the reference's rules."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import content_hash as och

GOLD = Path(__file__).parent / "golden" / "xxh64_vectors.npz"


def _vectors():
    z = np.load(GOLD)
    for i, n in enumerate(z["lengths"]):
        b = z["data"][z["offsets"][i]:z["offsets"][i] + n].tobytes()
        for j, s in enumerate(z["seeds"]):
            yield b, int(s), int(z["digests"][i, j])


def test_oracle_xxh64_matches_xxhash_vectors():
    for b, seed, d in _vectors():
        assert och.xxh64(b, seed) == d, (len(b), seed)


def test_library_xxh64_matches_xxhash_vectors(cuda_lib):
    from vlcache_b200 import ops
    for b, seed, d in _vectors():
        assert ops.xxh64(b, seed) == d, (len(b), seed)


@pytest.mark.parametrize("n", [0, 1, 31, 1023, 1024, 1025, 65536, 65537, 131075, 1 << 20, 8519757])
@pytest.mark.parametrize("hlen", [0, 3, 24, 256])
def test_host_tree_hash_matches_oracle(cuda_lib, n, hlen):
    from vlcache_b200 import ops
    rng = np.random.default_rng(n + hlen)
    data = rng.integers(0, 256, n, dtype=np.uint8)
    header = rng.integers(0, 256, hlen, dtype=np.uint8).tobytes()
    assert ops.content_hash(data, header) == och.tree_hash(data, header)
    assert ops.content_hash(data, header, num_threads=1) == och.tree_hash(data, header)


def test_tree_hash_separates_contents(cuda_lib):
    from vlcache_b200 import ops
    rng = np.random.default_rng(7)
    data = rng.integers(0, 256, 300000, dtype=np.uint8)
    base = ops.content_hash(data, b"grid")
    flipped = data.copy()
    flipped[123457] ^= 1
    assert ops.content_hash(flipped, b"grid") != base
    assert ops.content_hash(data, b"grie") != base
    assert ops.content_hash(data[:-1], b"grid") != base
    with pytest.raises(Exception):
        ops.content_hash(data, bytes(257))


def test_compute_hash_and_cache_policy(cuda_lib):
    """compute_hash keys an image by grid_thw (int64 header) + pixel bytes; the manager
    allocates, hits, refreshes and evicts least-recently-used entries as the reference."""
    from vlcache_b200.engine.encoder_cache import EncoderCacheManager, compute_hash
    g = torch.Generator().manual_seed(1)
    px = torch.randn(64, 1176, generator=g)
    grid = torch.tensor([1, 8, 8])
    key = compute_hash(px, grid)
    assert key == och.tree_hash(px.numpy().view(np.uint8), np.array([1, 8, 8], np.int64).tobytes())
    assert compute_hash(px.clone(), grid.clone()) == key and compute_hash(px, torch.tensor([1, 4, 16])) != key
    m = EncoderCacheManager(4, 16, 8, torch.float32, device="cpu")
    assert m.get_block_ids(1) is None
    a = m.allocate(1, 20)                      # 2 blocks
    b = m.allocate(2, 16)                      # 1 block
    assert len(a) == 2 and len(b) == 1 and m.allocate(1, 20) == a
    m.get_block_ids(1)                         # 1 becomes most recent
    c = m.allocate(3, 32)                      # needs 2: evicts 2 (least recent)
    assert m.get_block_ids(2) is None and m.get_block_ids(1) == a and len(c) == 2
    emb = torch.randn(20, 8, generator=g)
    m.write(a, emb)
    assert torch.equal(m.read(a, 20), emb)
    assert m.allocate(9, 16 * 5) is None       # larger than the whole cache
