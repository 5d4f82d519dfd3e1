"""CPU checks of bench.py's host-only legs (no GPU): the reference arm's sampler always
times at least one layer (its warm-up passes a zero budget)."""
import bench


def test_cpu_reference_sample_zero_budget_times_one_layer():
    value, layers, seconds, threads = bench.cpu_reference_sample(budget_s=0.0)
    assert layers == 1 and seconds > 0 and value > 0 and threads >= 1
