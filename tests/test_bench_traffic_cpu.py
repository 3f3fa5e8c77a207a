"""bench.py's roofline `traffic` lookup: every GPU count the driver runs
(1, 2, 4, 8) finds the per-launch DRAM bytes of the dominant kernel in a
committed ncu summary, and the figure is close to the algorithmic KV read of
that rank (2 * 64 * 8193 * kv_heads_per_rank * 128 * 2 bytes)."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_traffic_recorded_for_every_gpu_count(world):
    t = bench.profile_traffic(bench.traffic_key("decoder_stack_decode", world))
    assert t is not None
    algorithmic = 2 * 64 * 8193 * (8 // world) * 128 * 2
    assert 1.0 <= t / algorithmic < 1.05


def test_traffic_key_distinguishes_gpu_counts():
    keys = {bench.traffic_key("decoder_stack_decode", n) for n in (1, 2, 4, 8)}
    assert len(keys) == 4
    assert bench.profile_traffic("no_such_workload@n3") is None
