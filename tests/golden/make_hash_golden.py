"""Generate tests/golden/xxh64_vectors.npz: XXH64 digests computed by the ``xxhash``
package (the library the reference hashes with, nanovllm/engine/encoder_cache_manager.py:24-29)
over seeded random byte strings of tail-exercising lengths and several seeds.  The
oracle's and the library's XXH64 primitive are checked against these vectors.

Usage: python tests/golden/make_hash_golden.py   (needs the ``xxhash`` package)
"""
from pathlib import Path

import numpy as np
import xxhash

LENGTHS = [0, 1, 3, 4, 5, 7, 8, 9, 15, 16, 17, 31, 32, 33, 63, 64, 65, 100, 127, 1023, 1024, 1025, 4096, 10007]
SEEDS = [0, 1, 2, 3, 0xFFFFFFFFFFFFFFFF, 0x9E3779B185EBCA87]


def main():
    rng = np.random.default_rng(2024)
    data = rng.integers(0, 256, size=sum(LENGTHS), dtype=np.uint8)
    offsets = np.cumsum([0] + LENGTHS)
    digests = np.zeros((len(LENGTHS), len(SEEDS)), np.uint64)
    for i, n in enumerate(LENGTHS):
        b = data[offsets[i]:offsets[i] + n].tobytes()
        for j, s in enumerate(SEEDS):
            digests[i, j] = xxhash.xxh64(b, seed=s).intdigest()
    out = Path(__file__).with_name("xxh64_vectors.npz")
    np.savez_compressed(out, data=data, offsets=offsets, lengths=np.array(LENGTHS, np.int64),
                        seeds=np.array(SEEDS, np.uint64), digests=digests, xxhash_version=xxhash.VERSION)
    print(out)


if __name__ == "__main__":
    main()
