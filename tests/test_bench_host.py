"""CPU: the bench's host-memory plan for the e2e host tier. Every rank of a
box must reach the same plan (their schedules must agree), and the plan must
keep all ranks' page-locked tiers inside 60 % of the box's memory."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402

GB = 1_000_000_000


def _per_rank_bytes(mult, tier, pool_blocks=1024):
    if tier == "pool":
        return pool_blocks * bench.BLOCK_BYTES
    return (mult * bench.SLOTS + bench.TURNOVER + pool_blocks) * bench.BLOCK_BYTES


def test_plan_keeps_the_full_scene_when_memory_allows():
    for world, limit in ((1, 196 * GB), (2, 251 * GB), (8, 1056 * GB)):
        assert bench.plan_host_pool(world, "cache", 1024, limit) == (4, "cache")


def test_plan_shrinks_the_scene_then_falls_back_to_the_pool():
    for world in (1, 2, 4, 8):
        for limit in (60 * GB, 196 * GB, 251 * GB, 500 * GB, 1056 * GB):
            mult, tier = bench.plan_host_pool(world, "cache", 1024, limit)
            assert mult in (2, 3, 4) and tier in ("cache", "pool")
            if tier == "cache":
                assert world * _per_rank_bytes(mult, tier) <= 0.6 * limit
                bigger = mult + 1
                if bigger <= 4:
                    assert world * _per_rank_bytes(bigger, tier) > 0.6 * limit
    assert bench.plan_host_pool(8, "cache", 1024, 196 * GB) == (4, "pool")
    assert bench.plan_host_pool(8, "cache", 1024, 500 * GB) == (3, "cache")
    assert bench.plan_host_pool(4, "pool", 1024, 10 * GB) == (4, "pool")


def test_memory_limit_is_read_the_same_way_on_every_call():
    a, b = bench.host_memory_limit(), bench.host_memory_limit()
    assert a == b and a > 0
