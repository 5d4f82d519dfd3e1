"""Request sharding across GPUs (one process per GPU, no collective on the data path).

Warm requests are independent: each GPU owns its own paged KV cache and runs the
attention path for the requests dealt to it.  The deal is deterministic and computed
identically on every rank from host metadata, so ranks never exchange request data:
longest-processing-time-first by an attention cost estimate (query rows x visible keys),
ties broken by request index.
"""
from __future__ import annotations

import heapq

import numpy as np


def attention_cost(num_query_rows: int, num_keys: int) -> float:
    """Causal work of one request's query rows over its keys (query-key pairs, bottom-right aligned)."""
    q, k = int(num_query_rows), int(num_keys)
    return float((2 * k - q + 1) * q // 2) if q > 0 else 0.0


def shard_requests(costs, world_size: int) -> list[list[int]]:
    """Assign request indices to ranks, balancing the summed cost (LPT)."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    costs = np.asarray(costs, dtype=np.float64)
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world_size)]
    shards: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    return [sorted(s) for s in shards]


def local_requests(costs, rank: int, world_size: int) -> list[int]:
    """The request indices rank `rank` serves."""
    return shard_requests(costs, world_size)[rank]
