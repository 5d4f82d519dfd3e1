"""Encoder cache keyed by a content hash, drop-in for nanovllm/engine/encoder_cache_manager.py.

``EncoderCacheManager`` keeps the reference's interface and policy (block pool of
``[num_blocks, block_size, hidden]``, LRU ``OrderedDict`` from image hash to blocks,
``get_block_ids`` / ``allocate`` / ``read`` / ``write``, encoder_cache_manager.py:6-80).
What changes is ``compute_hash`` (:24-29): the reference runs XXH64 over the image's
``grid_thw`` bytes and its pixel bytes on the host, after copying a device tensor back,
about 198 MB per 4K image per request.  Here the key is this library's tree of XXH64
(``vlc_content_hash_*``): hashed in place on the GPU when the pixels are there (HBM
bandwidth, no copy), or over all host threads when they are on the host.  The keys are
only compared with each other inside one engine, so the change keeps the reference's
behaviour: identical grid and pixel bytes give the same key.
"""
from __future__ import annotations

from collections import OrderedDict, deque

import numpy as np
import torch

from .. import ops


def compute_hash(pixel_values_slice: torch.Tensor, grid_thw_item: torch.Tensor) -> int:
    """Key of one image: the tree hash of its pixel bytes with the int64 ``grid_thw`` as
    header (the reference hashes the same bytes in the same order)."""
    header = np.asarray(grid_thw_item.detach().cpu().numpy(), dtype=np.int64).tobytes()
    px = pixel_values_slice.detach()
    if not px.is_contiguous():
        px = px.contiguous()
    return ops.content_hash(px, header)


class EncoderCacheManager:
    """The reference's encoder cache (encoder_cache_manager.py:6-80) with ``compute_hash``
    replaced; block storage, LRU eviction and read/write are the same operations."""

    def __init__(self, num_blocks: int, block_size: int, hidden_size: int, dtype: torch.dtype,
                 device: torch.device | str = "cuda"):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.hidden_size = hidden_size
        self.dtype = dtype
        self.device = device
        self.free_block_ids = deque(range(num_blocks))
        self.hash_to_blocks: OrderedDict[int, list[int]] = OrderedDict()
        self.cache = torch.empty(num_blocks, block_size, hidden_size, dtype=dtype, device=device)

    compute_hash = staticmethod(compute_hash)

    def can_allocate(self, num_tokens: int) -> bool:
        return self.num_blocks >= (num_tokens + self.block_size - 1) // self.block_size

    def get_block_ids(self, hash_key: int):
        if hash_key in self.hash_to_blocks:
            self.hash_to_blocks.move_to_end(hash_key)
            return self.hash_to_blocks[hash_key]
        return None

    def allocate(self, hash_key: int, num_tokens: int) -> list[int] | None:
        if hash_key in self.hash_to_blocks:
            self.hash_to_blocks.move_to_end(hash_key)
            return self.hash_to_blocks[hash_key]
        needed = (num_tokens + self.block_size - 1) // self.block_size
        while len(self.free_block_ids) < needed:
            if not self.hash_to_blocks:
                return None   # one image larger than the whole cache
            _, blocks = self.hash_to_blocks.popitem(last=False)
            self.free_block_ids.extend(blocks)
        blocks = [self.free_block_ids.popleft() for _ in range(needed)]
        self.hash_to_blocks[hash_key] = blocks
        return blocks

    def read(self, block_ids: list[int], length: int) -> torch.Tensor:
        return self.cache[block_ids].reshape(-1, self.hidden_size)[:length]

    def write(self, block_ids: list[int], tensor: torch.Tensor) -> None:
        n = tensor.shape[0]
        flat = self.cache[block_ids].view(-1, self.hidden_size)
        flat[:n] = tensor
        flat[n:] = 0
        self.cache[block_ids] = flat.view(len(block_ids), self.block_size, self.hidden_size)
