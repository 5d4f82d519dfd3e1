"""CPU checks of bench.py's host-only legs (no GPU): the reference arm's sampler always
times at least one layer (its warm-up passes a zero budget)."""
import bench


def test_cpu_reference_sample_zero_budget_times_one_layer():
    value, layers, seconds, threads = bench.cpu_reference_sample(budget_s=0.0)
    assert layers == 1 and seconds > 0 and value > 0 and threads >= 1


def test_sharded_legs_cover_every_request_once():
    """cfg3's 64 requests and cfg5's 256 sequences are dealt to 1/2/4/8 ranks: each
    request lands on exactly one rank, and the largest share's cost is within 10 % of
    the mean (64 requests of similar cost over at most 8 ranks)."""
    import numpy as np

    from vlcache_b200.engine.sharding import attention_cost, shard_requests
    reqs, _, _, _ = bench.cfg3_requests()
    costs = [attention_cost(r.img_start + r.num_recompute, r.img_start + r.num_recompute) +
             attention_cost(r.seqlen - r.img_end, r.seqlen) for r in reqs]
    lens = np.random.default_rng(5).integers(2700, 10701, size=bench.DEC_SEQS)
    for world in (1, 2, 4, 8):
        for c in (costs, lens):
            shards = shard_requests(c, world)
            assert sorted(i for s in shards for i in s) == list(range(len(c)))
            loads = [sum(float(c[i]) for i in s) for s in shards]
            assert max(loads) <= 1.10 * (sum(loads) / world)
        total = sum(len(bench.cfg3_shard(r, world)[0]) for r in range(world))
        assert total == 64
