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
from tidegs_b200.sharded import BlockGradExchange, make_plan, owner_of


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
