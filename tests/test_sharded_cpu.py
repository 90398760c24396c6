"""CPU: the multi-GPU exchange plan and a real world-size-2 exchange over
gloo (host logic of tidegs_b200/sharded.py; the owner-side sum is the oracle
restatement here, the CUDA kernel in tests/test_gpu_sharded.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import blocks as ob
from tidegs_b200.sharded import (BlockGradExchange, exchange_arena_tables, make_gather_plan,
                                 make_plan, owner_of)


def test_plan_groups_by_owner_and_keeps_sender_order():
    vis = [[5, 0, 3, 4, 8], [3, 4, 1, 6], [8, 7, 4, 3]]
    W = 3
    plans = [make_plan(vis, W, r, block_size=2) for r in range(W)]
    # rank 0 sends its blocks grouped by owner (0: 0,3 | 1: 4 | 2: 5,8)
    assert plans[0].send_blocks.tolist() == [0, 3, 4, 5, 8]
    assert plans[0].send_counts == [2, 1, 2]
    # owner 1 receives 4 (from rank 0), 1,4 (rank 1), 4,7 (rank 2)
    p1 = plans[1]
    assert p1.recv_counts == [1, 2, 2]
    assert p1.recv_blocks.tolist() == [4, 1, 4, 4, 7]
    assert p1.out_blocks.tolist() == [1, 4, 7]
    # block 4's contributions in sender order: tiles 0 (rank 0), 2 (rank 1), 3 (rank 2)
    k = p1.out_blocks.tolist().index(4)
    assert p1.contrib_blocks[p1.contrib_offsets[k]:p1.contrib_offsets[k + 1]].tolist() == [0, 2, 3]
    # totals are consistent across ranks
    for r in range(W):
        for s in range(W):
            assert plans[s].send_counts[r] == plans[r].recv_counts[s]
    assert owner_of([0, 5, 7], 3).tolist() == [0, 2, 1]


def test_plan_output_order_follows_owner_rows():
    vis = [[2, 6, 4], [4, 0]]
    plan = make_plan(vis, 2, 0, block_size=1, out_order={0: 30, 2: 10, 4: 20, 6: 0})
    assert plan.out_blocks.tolist() == [6, 2, 4, 0]
    with pytest.raises(KeyError):
        make_plan(vis, 2, 0, block_size=1, out_order={0: 1})


@pytest.mark.parametrize("W", [2, 3, 5, 8])
def test_push_destinations_match_all_to_all_delivery(W):
    """send_dst_tiles puts every tile where all_to_all_single delivers it
    (sender-major, ascending block ids inside a sender)."""
    rng = np.random.default_rng(W)
    vis = [np.unique(rng.choice(300, 70, replace=False)) for _ in range(W)]
    vis[W - 1] = np.zeros(0, np.int64)  # a rank that rendered nothing
    plans = [make_plan(vis, W, r, block_size=1) for r in range(W)]
    for o in range(W):
        delivered = []
        for pl in plans:
            off = np.concatenate([[0], np.cumsum(pl.send_counts)])
            delivered += pl.send_blocks[off[o]:off[o + 1]].tolist()
        assert delivered == plans[o].recv_blocks.tolist()
        pushed = np.full(len(delivered), -1)
        for pl in plans:
            mine = owner_of(pl.send_blocks, W) == o
            assert np.all(pushed[pl.send_dst_tiles[mine]] == -1)  # no tile written twice
            pushed[pl.send_dst_tiles[mine]] = pl.send_blocks[mine]
        assert pushed.tolist() == delivered


@pytest.mark.parametrize("W", [2, 4, 7])
def test_pull_sources_point_at_each_senders_rows(W):
    """recv_src_tiles[t] is the row tile of received block t in its sender's
    gradients (the sender's rendered blocks in ascending id): the pull kernel
    reads contribution j of out block k from sender s at that tile."""
    rng = np.random.default_rng(30 + W)
    vis = [np.unique(rng.choice(200, 50, replace=False)) for _ in range(W)]
    for owner in range(W):
        plan = make_plan(vis, W, owner, block_size=1)
        sender = np.repeat(np.arange(W), plan.recv_counts)
        for t, b in enumerate(plan.recv_blocks.tolist()):
            rendered = np.unique(vis[sender[t]])
            assert rendered[plan.recv_src_tiles[t]] == b
        for k, b in enumerate(plan.out_blocks.tolist()):
            cs = plan.contrib_blocks[plan.contrib_offsets[k]:plan.contrib_offsets[k + 1]]
            ranks = sender[cs].tolist()
            assert ranks == sorted(ranks)  # summation in rank order
            assert ranks == [r for r in range(W) if b in set(vis[r].tolist())]


def test_plan_accepts_dense_order_table():
    vis = [[2, 6, 4], [4, 0]]
    table = np.full(10, -1, np.int64)
    table[[0, 2, 4, 6]] = [30, 10, 20, 0]
    plan = make_plan(vis, 2, 0, block_size=1, out_order=table)
    assert plan.out_blocks.tolist() == [6, 2, 4, 0]
    table[0] = -1
    with pytest.raises(KeyError):
        make_plan(vis, 2, 0, block_size=1, out_order=table)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tiles_for(rank, blocks, B):
    """Deterministic gradient tile of (rank, block): [B, 59] UNIFIED."""
    out = {}
    for b in blocks:
        rng = np.random.default_rng(1000 * rank + int(b))
        out[int(b)] = rng.standard_normal((B, 59)).astype(np.float32) * np.float32(1e-3)
    return out


def _worker(rank, world, port, vis, B, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = make_plan(vis, world, rank, B)
        tiles = _tiles_for(rank, plan.send_blocks, B)
        send = torch.from_numpy(np.concatenate([tiles[int(b)] for b in plan.send_blocks])
                                if plan.send_blocks.size else np.zeros((0, 59), np.float32))
        ex = BlockGradExchange(B)
        recv = ex.all_to_all(plan, send)
        got = ob.block_grad_sum(recv.numpy(), plan.contrib_offsets, plan.contrib_blocks, B)
        result_q.put((rank, plan.out_blocks.tolist(), {k: v.tolist() for k, v in got.items()}))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_exchange_equals_single_process_sum():
    world, B = 2, 4
    rng = np.random.default_rng(3)
    vis = [sorted(set(rng.integers(0, 40, 15).tolist())) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, vis, B, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, out_blocks, got = q.get(timeout=120)
        results[rank] = (out_blocks, got)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # single-process reference: every block's tiles summed in rank order
    for owner in range(world):
        out_blocks, got = results[owner]
        owned = sorted(b for b in set(vis[0]) | set(vis[1]) if b % world == owner)
        assert out_blocks == owned
        for k, b in enumerate(owned):
            s = None
            for r in range(world):
                if b in vis[r]:
                    t = _tiles_for(r, [b], B)[b]
                    s = t.copy() if s is None else (s + t).astype(np.float32)
            for name, w in ob.WIDTHS.items():
                col = ob.UNIFIED[name]
                np.testing.assert_array_equal(np.asarray(got[name], np.float32)[k * B:(k + 1) * B],
                                              s[:, col:col + w])


def _arena(world, owner, slots, pool, rng):
    """A rank's arena table: `slots` slots, some free, holding blocks it owns."""
    owned = np.arange(owner, pool, world, dtype=np.int64)
    held = rng.choice(owned, min(owned.size, slots - slots // 4), replace=False)
    table = np.full(slots, -1, np.int64)
    table[rng.choice(slots, held.size, replace=False)] = held
    return table


@pytest.mark.parametrize("W", [2, 3, 8])
def test_gather_plan_splits_own_remote_and_missing(W):
    rng = np.random.default_rng(W)
    pool, slots = 300, 40
    arenas = [_arena(W, o, slots, pool, rng) for o in range(W)]
    for me in range(W):
        want = rng.choice(pool, 60, replace=False)
        plan = make_gather_plan(want, arenas, W, me, 16)
        got = np.concatenate([plan.own_blocks, plan.remote_blocks, plan.missing])
        assert np.array_equal(np.sort(got), np.unique(want))
        assert np.all(plan.own_blocks % W == me)
        assert np.all(arenas[me][plan.own_slots] == plan.own_blocks)
        assert np.all(np.diff(plan.remote_blocks) > 0)
        assert np.all(plan.owner == plan.remote_blocks % W) and np.all(plan.owner != me)
        for b, o, sl in zip(plan.remote_blocks, plan.owner, plan.src_slot):
            assert arenas[o][sl] == b
        for b in plan.missing:
            assert b not in arenas[b % W]
        assert plan.owner_order() == [(me + d) % W for d in range(1, W)]


def test_gather_plan_rejects_an_arena_that_breaks_ownership():
    good = np.array([0, 2, -1, 4], np.int64)
    with pytest.raises(ValueError, match="does not own"):
        make_gather_plan([1], [good, np.array([1, 2, -1], np.int64)], 2, 0, 4)
    with pytest.raises(ValueError, match="twice"):
        make_gather_plan([1], [good, np.array([1, 3, 1], np.int64)], 2, 0, 4)
    with pytest.raises(ValueError, match="one arena table per rank"):
        make_gather_plan([1], [good], 2, 0, 4)


def _block_rows(b, B):
    """Deterministic parameter rows of block b: [B, 59] UNIFIED."""
    return np.random.default_rng(50_000 + int(b)).standard_normal((B, 59)).astype(np.float32)


def _gather_worker(rank, world, port, arenas, want, B, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = arenas[rank]
        data = np.zeros((mine.size * B, 59), np.float32)
        for s, b in enumerate(mine):
            if b >= 0:
                data[s * B:(s + 1) * B] = _block_rows(b, B)
        tables = exchange_arena_tables(mine[: mine.size - rank], "cpu")  # ragged tables
        plan = make_gather_plan(want[rank], tables, world, rank, B)
        # the copies PeerParamGather makes, with every rank's arena fetched here
        all_data = [torch.empty((a.size * B, 59)) for a in arenas]
        dist.all_gather(all_data, torch.from_numpy(data))
        render = np.zeros((plan.remote_blocks.size * B, 59), np.float32)
        for i, (o, sl) in enumerate(zip(plan.owner, plan.src_slot)):
            render[i * B:(i + 1) * B] = all_data[o].numpy()[sl * B:(sl + 1) * B]
        ok = all(np.array_equal(render[i * B:(i + 1) * B], _block_rows(b, B))
                 for i, b in enumerate(plan.remote_blocks))
        ok = ok and all(np.array_equal(t, a[: a.size - r])
                        for r, (t, a) in enumerate(zip(tables, arenas)))
        result_q.put((rank, ok, plan.remote_blocks.tolist(), plan.missing.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_param_gather_host_logic():
    """Arena tables all-gathered over gloo (ragged lengths) give every rank a
    gather plan whose copies deliver each remote block's owner rows."""
    world, B, pool, slots = 2, 4, 60, 24
    rng = np.random.default_rng(11)
    arenas = [_arena(world, o, slots, pool, rng) for o in range(world)]
    want = [np.sort(rng.choice(pool, 25, replace=False)) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, arenas, want, B, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, ok, remote, missing = q.get(timeout=120)
        results[rank] = (ok, remote, missing)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        ok, remote, missing = results[r]
        assert ok
        tables = [a[: a.size - o] for o, a in enumerate(arenas)]
        assert remote == [int(b) for b in want[r] if b % world != r and b in tables[b % world]]
        assert missing == [int(b) for b in want[r] if b not in tables[b % world]]
