"""CPU: the bench's host-side workload logic. Every rank of a box must derive
the same schedule and host-tier plan from the same inputs; the configs[4]
trajectory must give every owner exactly the configured turnover and ~30 %
of its slots visible, with neighbouring cameras sharing 70 % of their
blocks; the host-tier plan must keep all ranks' page-locked tiers inside
60 % of the box's memory."""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402

GB = 1_000_000_000


def test_host_tier_plan_fits_or_falls_back():
    for world in (1, 2, 4, 8):
        blocks = bench.Schedule(0, world).touched_blocks(15).size
        for limit in (60 * GB, 196 * GB, 500 * GB, 1056 * GB):
            tier = bench.plan_host_tier(world, "cache", 256, blocks, limit)
            need = world * (blocks + bench.TURNOVER + 256) * bench.BLOCK_BYTES
            assert tier == ("cache" if need <= 0.6 * limit else "pool")
    assert bench.plan_host_tier(4, "pool", 256, 10, 10 * GB) == "pool"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_trajectory_turnover_visibility_and_overlap(world):
    traj = bench.Trajectory(world)
    scheds = [bench.Schedule(r, world, traj) for r in range(world)]
    cams = traj.cameras(0)
    assert len(cams) == bench.CAMERAS
    overlap = (cams[0][1] - cams[1][0]) / traj.cam
    assert abs(overlap - bench.OVERLAP) < 0.02
    for k in range(40):
        vis = traj.visible(k)
        a = traj.start(k)
        assert a <= vis[0] and vis[-1] < a + traj.span  # the batch is resident
        rendered = bench.rendered_blocks(traj, k, world)
        assert np.array_equal(np.unique(np.concatenate(rendered)), vis)
        for r, sc in enumerate(scheds):
            pos = sc.visible_positions(k)
            assert abs(pos.size - bench.VISIBLE_FRAC * bench.SLOTS) <= 0.02 * bench.SLOTS
            assert np.all(sc.slot_block[pos] % world == r)
            ev, inc, dirty = sc.turnover(k)
            assert dirty is None
            assert ev.size == inc.size == bench.TURNOVER
            assert np.all(np.diff(ev) > 0) and np.all(np.diff(inc) > 0)
            assert not np.isin(inc, sc.slot_block).any()
            sc.slot_block[ev] = inc
            assert np.unique(sc.slot_block).size == bench.SLOTS
            assert np.all(sc.slot_block % world == r)


def test_trace_matches_a_fresh_replay_on_every_rank():
    world = 4
    traces = [bench.ScheduleTrace(world, r, 12) for r in range(world)]
    for k in range(12):
        for t in traces[1:]:
            for a, b in zip(t.vis[k], traces[0].vis[k]):
                assert np.array_equal(a, b)
    sched = bench.Schedule(2, world)
    for k in range(12):
        ev, inc, _ = sched.turnover(k)
        assert np.array_equal(ev, traces[2].turn[k][0])
        assert np.array_equal(inc, traces[2].turn[k][1])
        sched.slot_block[ev] = inc


def test_random_turnover_draws_non_resident_blocks():
    slot_block = np.arange(0, 64, dtype=np.int64)
    pool = np.arange(0, 256, dtype=np.int64)
    old = bench.TURNOVER
    bench.set_slots(64)
    try:
        rt = bench.RandomTurnover(slot_block, pool, seed=3)
        for k in range(5):
            ev, inc, dirty = rt.turnover(k)
            assert ev.size == inc.size == dirty.size == 16
            assert not np.isin(inc, slot_block).any()
            slot_block[ev] = inc
    finally:
        bench.set_slots(4 * old)


def test_memory_limit_is_read_the_same_way_on_every_call():
    a, b = bench.host_memory_limit(), bench.host_memory_limit()
    assert a == b and a > 0


@pytest.mark.parametrize("world", [2, 8])
def test_every_rendered_block_is_resident_at_its_owner(world):
    """The parameter gather needs no host-tier read: after step k's turnover
    every block a rank renders at step k+1 sits in its owner's slots."""
    from tidegs_b200.sharded import make_gather_plan

    traj = bench.Trajectory(world)
    scheds = [bench.Schedule(r, world, traj) for r in range(world)]
    for k in range(12):
        for sc in scheds:
            ev, inc, _ = sc.turnover(k)
            sc.slot_block[ev] = inc
        tables = [sc.slot_block for sc in scheds]
        for me in range(world):
            plan = make_gather_plan(traj.rendered(k + 1, me), tables, world, me, bench.B)
            assert plan.missing.size == 0
            assert plan.remote_blocks.size + plan.own_blocks.size == traj.rendered(k + 1, me).size
