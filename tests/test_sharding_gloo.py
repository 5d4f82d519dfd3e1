"""Multi-process (world_size 2, gloo on CPU) checks of the request-sharding host logic used
when the warm-prefill path runs one process per GPU (64 warm requests
sharing one image, prefix U[0,512], suffix U[16,128], ratio 0.05)."""
import math
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vlcache_b200.engine.sharding import attention_cost, local_requests, shard_requests


def cfg3_costs(seed=0, n=64):
    rng = np.random.default_rng(seed)
    n_img = 39 * 69
    R = math.ceil(0.05 * n_img)
    pre = rng.integers(0, 513, size=n)
    suf = rng.integers(16, 129, size=n)
    costs = []
    for p, s in zip(pre, suf):
        n_tok = p + n_img + s
        costs.append(attention_cost(p + R, p + R) + attention_cost(s, n_tok))
    return np.array(costs)


def test_shard_requests_partition_and_balance():
    costs = cfg3_costs()
    for world in (1, 2, 4, 8):
        shards = shard_requests(costs, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(costs)))
        loads = [costs[s].sum() for s in shards]
        assert max(loads) <= min(loads) + costs.max()   # LPT bound


def test_attention_cost_matches_causal_pairs():
    from oracle.attention import causal_pairs
    assert attention_cost(1075, 1075) + attention_cost(48, 10617) == causal_pairs([0, 1075, 1123], [0, 1075, 11692])


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = cfg3_costs()
        mine = local_requests(costs, rank, world)
        # every rank derives the same deal without exchanging request data; gather to check
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        # max-over-ranks reduction of a per-rank time, as bench.py does for its timing
        t = torch.tensor([float(len(mine) + rank)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(repr((gathered, float(t.item()))))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding(tmp_path):
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    res = [eval((tmp_path / f"rank{r}.txt").read_text()) for r in range(2)]
    assert res[0] == res[1]
    shards, tmax = res[0]
    assert sorted(shards[0] + shards[1]) == list(range(64))
    assert not set(shards[0]) & set(shards[1])
    assert tmax == max(len(shards[0]), len(shards[1]) + 1)
