"""GPU: the multi-GPU gradient exchange (tidegs_b200/sharded.py).

Parity definition (the reference is single-GPU): the owner's gradients and
Adam update after pack -> all-to-all -> ordered sum equal the single-GPU
result on the same per-rank gradients summed in rank order, bit for bit.
Ranks are emulated inside one process here (the all-to-all's delivery order
is reproduced by concatenation); test_two_gpu_nccl_exchange runs the real
NCCL exchange when the box has two GPUs. The direct push (tgs_grad_push,
PeerGradExchange) must put every tile exactly where the all-to-all puts it:
emulated here with every "peer" buffer on one GPU, and over CUDA IPC between
two GPUs in test_two_gpu_peer_push. The pull path (PeerGradPull +
GPUResidentAdam.step_pulled: the owner's update kernel sums the senders'
gradients itself) must equal exchange + sum + plain update bit for bit:
emulated ranks here, two GPUs in test_two_gpu_pull_sum_adam. The parameter
gather (PeerParamGather: updated blocks copied from their owners' arenas to
the ranks that render them next) must deliver every remote block's owner rows
bit for bit: emulated owners on one GPU, an owner on a second GPU in one
process, and two processes over CUDA IPC in test_two_gpu_param_gather."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import blocks as ob
from tidegs_b200 import _lib, _ops
from tidegs_b200.sharded import (BlockGradExchange, PeerGradExchange, PeerGradPull,
                                 PeerParamGather, exchange_arena_tables, make_gather_plan,
                                 make_plan, owner_of)

pytestmark = pytest.mark.gpu

NAMES = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")


def _compact_grads(rank, blocks, B):
    """SoA gradients of `blocks` (rows in listed order), seeded by (rank, block)."""
    tiles = []
    for b in blocks:
        rng = np.random.default_rng(7919 * rank + int(b))
        tiles.append(rng.standard_normal((B, 59)).astype(np.float32) * np.float32(1e-3))
    aos = np.concatenate(tiles) if tiles else np.zeros((0, 59), np.float32)
    return aos, {n: torch.from_numpy(aos[:, ob.UNIFIED[n]:ob.UNIFIED[n] + w].copy()).cuda()
                 for n, w in ob.WIDTHS.items()}


def _emulate(vis, W, B):
    """Send buffers of every rank, then each owner's receive buffer in the
    order all_to_all_single delivers it (sender 0's tiles first)."""
    ex = BlockGradExchange(B)
    plans = [make_plan(vis, W, r, B) for r in range(W)]
    sends = []
    for r, plan in enumerate(plans):
        order = sorted(int(b) for b in plan.send_blocks)  # rows of the rank's compact grads
        aos, soa = _compact_grads(r, order, B)
        start = {b: i * B for i, b in enumerate(order)}
        send = ex.pack(plan, soa, start)
        # the packed tiles are the rank's tiles in send order
        expect = np.concatenate([aos[start[int(b)]:start[int(b)] + B] for b in plan.send_blocks])
        np.testing.assert_array_equal(send.cpu().numpy(), expect)
        sends.append((plan, send))
    recvs = []
    for o in range(W):
        parts = []
        for s, (plan, send) in enumerate(sends):
            off = sum(plan.send_counts[:o]) * B
            parts.append(send[off: off + plan.send_counts[o] * B])
        recvs.append(torch.cat(parts) if parts else torch.empty((0, 59), device="cuda"))
    return ex, plans, recvs


@pytest.mark.parametrize("W,B", [(4, 64), (3, 16384)])
def test_ordered_block_sum_matches_oracle(W, B):
    rng = np.random.default_rng(W)
    nb = 96 if B == 64 else 12
    vis = [sorted(set(rng.integers(0, nb, nb // 2).tolist())) for _ in range(W)]
    ex, plans, recvs = _emulate(vis, W, B)
    for o in range(W):
        got = ex.reduce(plans[o], recvs[o])
        want = ob.block_grad_sum(recvs[o].cpu().numpy(), plans[o].contrib_offsets,
                                 plans[o].contrib_blocks, B)
        for n in NAMES:
            np.testing.assert_array_equal(got[n].cpu().numpy(), want[n], err_msg=n)


def test_owner_adam_after_exchange_equals_single_gpu():
    """Owner Adam on exchanged gradients == Adam on the rank-order sum."""
    import types

    from tidegs_b200 import GPUResidentAdam

    W, B = 3, 64
    rng = np.random.default_rng(9)
    vis = [sorted(set(rng.integers(0, 60, 25).tolist())) for _ in range(W)]
    ex, plans, recvs = _emulate(vis, W, B)
    owner = 1
    plan = plans[owner]
    owned = plan.out_blocks.tolist()
    rows = len(owned) * B
    layout = [(b, slice(i * B, (i + 1) * B)) for i, b in enumerate(owned)]
    params = {n: torch.randn((rows, w), device="cuda") for n, w in ob.WIDTHS.items()}
    ids = torch.arange(rows, device="cuda")

    def run(grads):
        class M:
            loaded_blocks = owned
            block_to_gpu_slice = dict(layout)
            local_to_global_idx = ids
        g = types.SimpleNamespace(gpu_working_set_manager=M(), optimizer=types.SimpleNamespace(
            columns_lr=torch.tensor([1e-3, 5e-2, 5e-3, 1e-3, 2.5e-3, 1e-4]),
            param_groups=[{"betas": (0.9, 0.999), "eps": 1e-15}]))
        for n in NAMES:
            setattr(g, "_" + n, params[n].clone())
        opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=len(owned))
        opt.set_resident_blocks(owned)
        opt.step(1, g, ids, grads)
        return {n: getattr(g, "_" + n).cpu() for n in NAMES}

    exchanged = ex.reduce(plan, recvs[owner])
    # single GPU: every rank's tiles of each owned block, summed in rank order
    summed = {n: torch.empty((rows, w), device="cuda") for n, w in ob.WIDTHS.items()}
    for k, b in enumerate(owned):
        s = None
        for r in range(W):
            if b in vis[r]:
                aos, _ = _compact_grads(r, [b], B)
                s = aos.copy() if s is None else (s + aos).astype(np.float32)
        for n, w in ob.WIDTHS.items():
            summed[n][k * B:(k + 1) * B] = torch.from_numpy(s[:, ob.UNIFIED[n]:ob.UNIFIED[n] + w].copy())
    a = run(exchanged)
    b = run(summed)
    for n in NAMES:
        assert torch.equal(a[n], b[n]), n


def _push_emulated(plans, soas, starts, recv_bufs, err=None):
    """Runs tgs_grad_push for every emulated rank, 'peer' buffers all local."""
    W = len(plans)
    for r, plan in enumerate(plans):
        n = int(plan.send_blocks.size)
        if n == 0:
            continue
        B = plan.block_size
        tab = torch.from_numpy(np.concatenate([starts[r], np.full(n, B, np.int64),
                                               plan.send_dst_tiles * B])).cuda()
        ranks = torch.from_numpy(owner_of(plan.send_blocks, W).astype(np.int32)).cuda()
        a = _lib.GradPushArgs()
        for c, n_ in enumerate(NAMES):
            a.comp[c] = soas[r][n_].data_ptr()
        a.src_start, a.row_count = tab[:n].data_ptr(), tab[n:2 * n].data_ptr()
        a.dst_row, a.dst_rank = tab[2 * n:].data_ptr(), ranks.data_ptr()
        a.n_tiles, a.max_rows, a.n_ranks = n, B, W
        for o in range(W):
            a.recv[o] = recv_bufs[o].data_ptr()
            a.recv_rows[o] = recv_bufs[o].shape[0]
        a.err = _lib.ptr(err)
        _lib.call("tgs_grad_push", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()


@pytest.mark.parametrize("W,B", [(4, 64), (3, 16384), (2, 100)])
def test_push_lands_where_all_to_all_delivers(W, B):
    rng = np.random.default_rng(11 + W)
    nb = 80 if B != 16384 else 12
    vis = [sorted(set(rng.integers(0, nb, nb // 2).tolist())) for _ in range(W)]
    ex, plans, recvs = _emulate(vis, W, B)
    soas, starts = [], []
    for r, plan in enumerate(plans):
        order = sorted(int(b) for b in plan.send_blocks)
        soas.append(_compact_grads(r, order, B)[1])
        starts.append(np.searchsorted(order, plan.send_blocks).astype(np.int64) * B)
    cap = [max(1, sum(pl.recv_counts)) * B + 3 for pl in plans]  # slack rows stay untouched
    bufs = [torch.full((c, 59), -7.0, device="cuda") for c in cap]
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    _push_emulated(plans, soas, starts, bufs, err)
    assert err.cpu().tolist() == [0, 0, 0, 0]
    for o in range(W):
        n = recvs[o].shape[0]
        assert torch.equal(bufs[o][:n], recvs[o]), o
        assert bool((bufs[o][n:] == -7.0).all())
        got = ex.reduce(plans[o], bufs[o][:n])
        want = ob.block_grad_sum(recvs[o].cpu().numpy(), plans[o].contrib_offsets,
                                 plans[o].contrib_blocks, B)
        for n_ in NAMES:
            np.testing.assert_array_equal(got[n_].cpu().numpy(), want[n_], err_msg=n_)


def test_push_reports_tile_outside_receive_buffer():
    W, B = 2, 64
    vis = [[0, 1, 2, 3], [1, 2]]
    plans = [make_plan(vis, W, r, B) for r in range(W)]
    soas, starts = [], []
    for r, plan in enumerate(plans):
        order = sorted(int(b) for b in plan.send_blocks)
        soas.append(_compact_grads(r, order, B)[1])
        starts.append(np.searchsorted(order, plan.send_blocks).astype(np.int64) * B)
    # owner 1 receives 3 tiles (blocks 1, 3 from rank 0, block 1 from rank 1);
    # give it room for 2: rank 1's tile (its send tile 1, destination tile 2)
    # must be skipped and reported, the two that fit written
    assert plans[1].recv_counts == [2, 1]
    bufs = [torch.zeros((sum(pl.recv_counts) * B, 59), device="cuda") for pl in plans]
    bufs[1] = torch.zeros((2 * B, 59), device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    _push_emulated(plans, soas, starts, bufs, err)
    code, idx_lo, _, aux = err.cpu().tolist()
    assert (code, idx_lo, aux) == (5, 1, 1)  # TGS_DEV_BAD_SLICE, tile 1, owner 1
    want = np.concatenate([_compact_grads(0, [1], B)[0], _compact_grads(0, [3], B)[0]])
    np.testing.assert_array_equal(bufs[1].cpu().numpy(), want)


def test_peer_exchange_single_rank_equals_all_to_all_path():
    W, B = 1, 256
    vis = [[3, 5, 8, 9]]
    plan = make_plan(vis, W, 0, B)
    order = sorted(int(b) for b in plan.send_blocks)
    _, soa = _compact_grads(0, order, B)
    starts = {b: i * B for i, b in enumerate(order)}
    ex = BlockGradExchange(B)
    want = ex.reduce(plan, ex.all_to_all(plan, ex.pack(plan, soa, starts)))
    peer = PeerGradExchange(B, capacity_blocks=8, device="cuda")
    try:
        for parity in (0, 1):
            assert peer.push(plan, soa, starts, parity) == 4 * B
            peer.barrier()
            got = peer.reduce(plan, parity)
            for n in NAMES:
                assert torch.equal(got[n], want[n]), n
    finally:
        peer.close()


LR6 = [1e-3, 5e-2, 5e-3, 1e-3, 2.5e-3, 1e-4]


def _owner(owned, B, params):
    """A GPUResidentAdam whose working set is `owned` (slice i = block i)."""
    import types

    from tidegs_b200 import GPUResidentAdam

    rows = len(owned) * B
    ids = torch.arange(rows, device="cuda")

    class M:
        loaded_blocks = list(owned)
        block_to_gpu_slice = {b: slice(i * B, (i + 1) * B) for i, b in enumerate(owned)}
        local_to_global_idx = ids

    g = types.SimpleNamespace(gpu_working_set_manager=M(), optimizer=types.SimpleNamespace(
        columns_lr=torch.tensor(LR6), param_groups=[{"betas": (0.9, 0.999), "eps": 1e-15}]))
    for n in NAMES:
        setattr(g, "_" + n, params[n].clone())
    opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=len(owned), device="cuda")
    opt.set_resident_blocks(list(owned))
    return opt, g


@pytest.mark.parametrize("W,B", [(3, 64), (2, 16384), (5, 32)])
def test_pull_sum_adam_equals_exchange_then_adam(W, B):
    rng = np.random.default_rng(40 + W)
    nb = 70 if B != 16384 else 10
    vis = [sorted(set(rng.integers(0, nb, nb // 2).tolist())) for _ in range(W)]
    ex, plans, recvs = _emulate(vis, W, B)
    # each rank's gradients: its rendered blocks in ascending id, B rows each
    grads = [_compact_grads(r, sorted(int(b) for b in plans[r].send_blocks), B)[1]
             for r in range(W)]
    for o in range(W):
        plan = plans[o]
        owned = plan.out_blocks.tolist()
        if not owned:
            continue
        params = {n: torch.randn((len(owned) * B, w), device="cuda") for n, w in ob.WIDTHS.items()}
        summed = ex.reduce(plan, recvs[o])
        opt_a, g_a = _owner(owned, B, params)
        opt_b, g_b = _owner(owned, B, params)
        pull = PeerGradPull.in_process(grads, o, B, "cuda")
        ids = torch.arange(len(owned) * B, device="cuda")
        for step in (1, 2, 3):
            sa = opt_a.step(step, g_a, ids, summed)
            sb = opt_b.step_pulled(step, g_b, ids, pull, plan)
            assert sa == sb
        for n in NAMES:
            assert torch.equal(getattr(g_a, "_" + n), getattr(g_b, "_" + n)), (o, n)
        assert torch.equal(opt_a._state, opt_b._state)


def test_pull_reads_a_sender_on_another_gpu_in_process():
    """One process, two GPUs: rank 1's gradients on cuda:1 are read over
    peer access by the owner's kernel on cuda:0; same result as the
    exchange + sum + plain update."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    W, B = 2, 64
    rng = np.random.default_rng(12)
    vis = [sorted(set(rng.integers(0, 40, 20).tolist())) for _ in range(W)]
    ex, plans, recvs = _emulate(vis, W, B)
    grads = [_compact_grads(r, sorted(int(b) for b in plans[r].send_blocks), B)[1]
             for r in range(W)]
    grads[1] = {n: t.to("cuda:1") for n, t in grads[1].items()}
    plan = plans[0]
    owned = plan.out_blocks.tolist()
    params = {n: torch.randn((len(owned) * B, w), device="cuda:0") for n, w in ob.WIDTHS.items()}
    summed = ex.reduce(plan, recvs[0])
    opt_a, g_a = _owner(owned, B, params)
    opt_b, g_b = _owner(owned, B, params)
    pull = PeerGradPull.in_process(grads, 0, B, "cuda:0")
    ids = torch.arange(len(owned) * B, device="cuda:0")
    for step in (1, 2):
        assert opt_a.step(step, g_a, ids, summed) == opt_b.step_pulled(step, g_b, ids, pull, plan)
    for n in NAMES:
        assert torch.equal(getattr(g_a, "_" + n), getattr(g_b, "_" + n)), n
    assert torch.equal(opt_a._state, opt_b._state)


def test_pull_rejects_rows_that_do_not_match_the_plan():
    W, B = 2, 32
    vis = [[0, 1], [1]]
    plans = [make_plan(vis, W, r, B) for r in range(W)]
    grads = [_compact_grads(r, sorted(int(b) for b in plans[r].send_blocks), B)[1]
             for r in range(W)]
    owned = plans[1].out_blocks.tolist()
    params = {n: torch.randn((len(owned) * B, w), device="cuda") for n, w in ob.WIDTHS.items()}
    opt, g = _owner(owned, B, params)
    pull = PeerGradPull.in_process(grads, 1, B, "cuda")
    with pytest.raises(ValueError):
        opt.step_pulled(1, g, torch.arange(B - 1, device="cuda"), pull, plans[1])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, vis, B, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        plan = make_plan(vis, world, rank, B)
        order = sorted(int(b) for b in plan.send_blocks)
        _, soa = _compact_grads(rank, order, B)
        ex = BlockGradExchange(B, device=torch.device("cuda", rank))
        send = ex.pack(plan, soa, {b: i * B for i, b in enumerate(order)})
        recv = ex.all_to_all(plan, send)
        got = ex.reduce(plan, recv)
        want = ob.block_grad_sum(recv.cpu().numpy(), plan.contrib_offsets, plan.contrib_blocks, B)
        ok = all(np.array_equal(got[n].cpu().numpy(), want[n]) for n in NAMES)
        # and the received tiles are exactly the senders' tiles
        expect = []
        for s in range(world):
            blocks = [b for b in np.unique(vis[s]) if b % world == rank]
            for b in blocks:
                aos, _ = _compact_grads(s, [int(b)], B)
                expect.append(aos)
        ok = ok and np.array_equal(recv.cpu().numpy(),
                                   np.concatenate(expect) if expect else np.zeros((0, 59), np.float32))
        torch.cuda.synchronize()
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_two_gpu_nccl_exchange():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, B = 2, 256
    rng = np.random.default_rng(5)
    vis = [sorted(set(rng.integers(0, 64, 30).tolist())) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, vis, B, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def _peer_worker(rank, world, port, vis_steps, B, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    peer = None
    try:
        cap = max(sum(make_plan(v, world, rank, B).recv_counts) for v in vis_steps)
        peer = PeerGradExchange(B, capacity_blocks=cap, device=torch.device("cuda", rank))
        ok = True
        for step, vis in enumerate(vis_steps):
            plan = make_plan(vis, world, rank, B)
            order = sorted(int(b) for b in plan.send_blocks)
            _, soa = _compact_grads(rank + 10 * step, order, B)
            peer.push(plan, soa, {b: i * B for i, b in enumerate(order)}, parity=step)
            peer.barrier()
            got = peer.reduce(plan, parity=step)
            expect = []
            for s in range(world):
                for b in (b for b in np.unique(vis[s]) if b % world == rank):
                    expect.append(_compact_grads(s + 10 * step, [int(b)], B)[0])
            recv = np.concatenate(expect) if expect else np.zeros((0, 59), np.float32)
            want = ob.block_grad_sum(recv, plan.contrib_offsets, plan.contrib_blocks, B)
            ok = ok and all(np.array_equal(got[n].cpu().numpy(), want[n]) for n in NAMES)
        torch.cuda.synchronize()
        q.put((rank, bool(ok)))
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


def test_two_gpu_peer_push():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, B = 2, 256
    rng = np.random.default_rng(6)
    vis_steps = [[sorted(set(rng.integers(0, 64, 30).tolist())) for _ in range(world)]
                 for _ in range(3)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, vis_steps, B, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def _pull_worker(rank, world, port, vis_steps, B, nb, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    pull = None
    try:
        cap = max(len(set(v[rank])) for v in vis_steps)
        grads = {n: torch.zeros((cap * B, w), device="cuda") for n, w in ob.WIDTHS.items()}
        pull = PeerGradPull(grads, B, torch.device("cuda", rank))
        owned = [b for b in range(nb) if b % world == rank]  # every block this rank owns
        table = np.full(nb, -1, np.int64)
        table[owned] = np.arange(len(owned))
        gen = torch.Generator(device="cuda").manual_seed(77 + rank)
        params = {n: torch.randn((len(owned) * B, w), device="cuda", generator=gen)
                  for n, w in ob.WIDTHS.items()}
        opt_a, g_a = _owner(owned, B, params)   # fused pull
        opt_b, g_b = _owner(owned, B, params)   # rank-order sum computed here, plain update
        ok = True
        for step, vis in enumerate(vis_steps, start=1):
            plan = make_plan(vis, world, rank, B, out_order=table)
            mine = sorted(int(b) for b in plan.send_blocks)
            _, soa = _compact_grads(rank + 10 * step, mine, B)
            for n in NAMES:
                grads[n][:len(mine) * B].copy_(soa[n])
            ids = torch.from_numpy((table[plan.out_blocks][:, None] * B
                                    + np.arange(B)[None, :]).reshape(-1)).cuda()
            sa = opt_a.step_pulled(step, g_a, ids, pull, plan)
            summed = {n: torch.empty((plan.n_out * B, w), device="cuda")
                      for n, w in ob.WIDTHS.items()}
            for k, b in enumerate(plan.out_blocks.tolist()):
                acc = None
                for r in range(world):
                    if b in vis[r]:
                        t = _compact_grads(r + 10 * step, [b], B)[0]
                        acc = t.copy() if acc is None else (acc + t).astype(np.float32)
                for n, w in ob.WIDTHS.items():
                    summed[n][k * B:(k + 1) * B] = torch.from_numpy(
                        acc[:, ob.UNIFIED[n]:ob.UNIFIED[n] + w].copy())
            sb = opt_b.step(step, g_b, ids, summed)
            ok = ok and sa == sb
        for n in NAMES:
            ok = ok and torch.equal(getattr(g_a, "_" + n), getattr(g_b, "_" + n))
        ok = ok and torch.equal(opt_a._state, opt_b._state)
        torch.cuda.synchronize()
        q.put((rank, bool(ok)))
    finally:
        if pull is not None:
            pull.close()
        dist.destroy_process_group()


def test_two_gpu_pull_sum_adam():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, B, nb = 2, 256, 40
    rng = np.random.default_rng(8)
    vis_steps = [[sorted(set(rng.integers(0, nb, 18).tolist())) for _ in range(world)]
                 for _ in range(3)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pull_worker, args=(r, world, port, vis_steps, B, nb, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


def _gather_arenas(world, slots, B, pool, seed, devices):
    """Per owner: arena table (block per slot, some free) and seeded arena
    component tensors on devices[owner]."""
    rng = np.random.default_rng(seed)
    tables, arenas = [], []
    for o in range(world):
        owned = np.arange(o, pool, world, dtype=np.int64)
        held = rng.choice(owned, min(owned.size, slots - 3), replace=False)
        t = np.full(slots, -1, np.int64)
        t[rng.choice(slots, held.size, replace=False)] = held
        tables.append(t)
        gen = torch.Generator(device=devices[o]).manual_seed(seed + o)
        arenas.append({n: torch.randn((slots * B, w), device=devices[o], generator=gen)
                       for n, w in ob.WIDTHS.items()})
    return tables, arenas


def _check_gathered(plan, arenas, render, B):
    for i, (o, sl) in enumerate(zip(plan.owner, plan.src_slot)):
        for n in NAMES:
            want = arenas[o][n][sl * B:(sl + 1) * B].to(render[n].device)
            assert torch.equal(render[n][i * B:(i + 1) * B], want), (i, n)


@pytest.mark.parametrize("W,B", [(3, 64), (4, 6)])
def test_param_gather_emulated_owners_bit_exact(W, B):
    """Owners emulated on one GPU; B = 6 puts odd slots off the 16-byte
    boundary, so the kernel's plain-copy path runs beside the bulk one."""
    slots, pool = 24, 120
    tables, arenas = _gather_arenas(W, slots, B, pool, 5 + W, ["cuda:0"] * W)
    rng = np.random.default_rng(W)
    for me in range(W):
        plan = make_gather_plan(rng.choice(pool, 50, replace=False), tables, W, me, B)
        assert plan.remote_blocks.size > 0
        gather = PeerParamGather.in_process(arenas, me, B, "cuda:0")
        render = {n: torch.full((plan.remote_blocks.size * B, w), float("nan"), device="cuda:0")
                  for n, w in ob.WIDTHS.items()}
        err = torch.zeros(4, dtype=torch.int32, device="cuda:0")
        assert gather.gather(render, plan, err=err) == plan.remote_blocks.size * B
        torch.cuda.synchronize()
        assert int(err[0].item()) == 0
        _check_gathered(plan, arenas, render, B)
        gather.close()


def test_param_gather_rejects_small_render_rows_and_foreign_plans():
    W, B = 2, 16
    tables, arenas = _gather_arenas(W, 8, B, 40, 3, ["cuda:0"] * W)
    plan = make_gather_plan(np.arange(40), tables, W, 0, B)
    gather = PeerParamGather.in_process(arenas, 0, B, "cuda:0")
    small = {n: torch.empty(((plan.remote_blocks.size - 1) * B, w), device="cuda:0")
             for n, w in ob.WIDTHS.items()}
    with pytest.raises(RuntimeError, match="the plan needs"):
        gather.launch(small, plan)
    other = make_gather_plan(np.arange(40), tables, W, 1, B)
    with pytest.raises(ValueError, match="another world/rank"):
        gather.tables(other)


def test_param_gather_reads_an_owner_on_another_gpu_in_process():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    W, B = 2, 256
    tables, arenas = _gather_arenas(W, 16, B, 64, 9, ["cuda:0", "cuda:1"])
    plan = make_gather_plan(np.arange(64), tables, W, 0, B)
    gather = PeerParamGather.in_process(arenas, 0, B, "cuda:0")
    render = {n: torch.empty((plan.remote_blocks.size * B, w), device="cuda:0")
              for n, w in ob.WIDTHS.items()}
    gather.gather(render, plan)
    torch.cuda.synchronize()
    _check_gathered(plan, arenas, render, B)


def _param_gather_worker(rank, world, port, B, slots, pool, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    gather = None
    try:
        dev = torch.device("cuda", rank)
        # every rank rebuilds all arenas' contents on the CPU to check against
        tables, arenas_cpu = _gather_arenas(world, slots, B, pool, 21, ["cpu"] * world)
        arena = {n: t.to(dev) for n, t in arenas_cpu[rank].items()}
        gather = PeerParamGather(arena, B, dev)
        got_tables = exchange_arena_tables(tables[rank], dev)
        ok = all(np.array_equal(a, b) for a, b in zip(got_tables, tables))
        want = np.random.default_rng(100 + rank).choice(pool, pool // 2, replace=False)
        plan = make_gather_plan(want, got_tables, world, rank, B)
        render = {n: torch.empty((max(1, plan.remote_blocks.size) * B, w), device=dev)
                  for n, w in ob.WIDTHS.items()}
        err = torch.zeros(4, dtype=torch.int32, device=dev)
        for _ in range(2):
            gather.gather(render, plan, err=err)
        torch.cuda.synchronize()
        ok = ok and int(err[0].item()) == 0 and plan.remote_blocks.size > 0
        for i, (o, sl) in enumerate(zip(plan.owner, plan.src_slot)):
            for n in NAMES:
                ok = ok and torch.equal(render[n][i * B:(i + 1) * B].cpu(),
                                        arenas_cpu[o][n][sl * B:(sl + 1) * B])
        q.put((rank, bool(ok)))
    finally:
        if gather is not None:
            gather.close()
        dist.destroy_process_group()


def test_two_gpu_param_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, B, slots, pool = 2, 1024, 24, 60
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_param_gather_worker, args=(r, world, port, B, slots, pool, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}
