"""GPU: the multi-GPU gradient exchange (tidegs_b200/sharded.py).

Parity definition (the reference is single-GPU): the owner's gradients and
Adam update after pack -> all-to-all -> ordered sum equal the single-GPU
result on the same per-rank gradients summed in rank order, bit for bit.
Ranks are emulated inside one process here (the all-to-all's delivery order
is reproduced by concatenation); test_two_gpu_nccl_exchange runs the real
NCCL exchange when the box has two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import blocks as ob
from tidegs_b200.sharded import BlockGradExchange, make_plan

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
