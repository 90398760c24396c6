"""GPU parity of the resident Adam kernels' staged (contiguous-chunk) paths.

The update kernels walk the touched rows in chunks of 32. A chunk whose 32 ids
are consecutive AND whose 32 state rows are consecutive -- every chunk of a
step that updates whole visible blocks, the benchmark's case -- is staged:
when its first id is a multiple of 4 the bulk-copy pipeline streams it (state
rows, parameters and gradients copied into shared memory, updated there and
copied back); otherwise the per-row kernel's staged branch brings its state
rows in by bulk copies while the parameters and gradients of the next rows
load into registers. Every other chunk (sparse rows) resolves and loads row
by row. All paths must give the reference's update: the kernel-order
restatement of
strategies/tide_engine/gpu_resident_optimizer.py:339-364 in
oracle/resident_adam.py, bit for bit, for parameters and both moments.

Cases (both the single-GPU kernel and the pull kernel that sums the senders'
gradients in rank order inside the update):
  * whole visible blocks (runs of blocks, all rows);
  * a short tail block in the middle of the working set (n not a multiple of
    32, chunks starting at unaligned rows);
  * blocks shorter than 32 rows whose slots are out of order, so that a
    chunk's ids are consecutive but its state rows are not -- including
    chunks whose first and last rows line up (slot order 0,5,2,3,4,1,6,7 of
    4-row blocks), which must NOT take the staged path;
  * block sizes that are not multiples of 32 (chunks crossing into the next
    position's slot, adjacent or not);
  * slots re-admitted after eviction and slots reused by another block: the
    stale rows' admission stamps must read as m = v = 0 on the staged path.

`_staged_chunks` restates the kernel's path choice on the host, so each test
also proves that its inputs drive the staged path (and, for the 4-row case,
that a first/last-only test would have mis-routed a chunk)."""
import types
import zlib

import numpy as np
import pytest
import torch

from oracle import blocks as ob
from oracle.resident_adam import COMPONENT_SPECS, ResidentAdamOracle

pytestmark = pytest.mark.gpu

NAMES = [n for n, _, _, _ in COMPONENT_SPECS]
ATTRS = {n: a for n, a, _, _ in COMPONENT_SPECS}
WIDTHS = {n: w for n, _, w, _ in COMPONENT_SPECS}
LRS = [1.6e-4, 0.05, 5e-3, 1e-3, 2.5e-3, 1.25e-4]
BETAS = (0.9, 0.999)
EPS = 1e-15


class _Manager:
    def __init__(self, layout):
        self.set_layout(layout)

    def set_layout(self, layout):
        self.loaded_blocks = [b for b, _ in layout]
        self.block_to_gpu_slice = {b: s for b, s in layout}
        self.local_to_global_idx = torch.arange(max(s.stop for _, s in layout), device="cuda")


def _gaussians(manager, params):
    g = types.SimpleNamespace(
        gpu_working_set_manager=manager,
        optimizer=types.SimpleNamespace(columns_lr=torch.tensor(LRS, dtype=torch.float32),
                                        param_groups=[{"betas": BETAS, "eps": EPS}]))
    for n in NAMES:
        setattr(g, ATTRS[n], torch.nn.Parameter(torch.from_numpy(params[n]).cuda().clone()))
    return g


def _values(g):
    return {n: getattr(g, ATTRS[n]).detach().cpu().numpy() for n in NAMES}


def _staged_chunks(ids, layout, block_to_slot, B):
    """(chunks the kernels stage, chunks a first/last-row-only test would
    stage, chunks the bulk-copy pipeline streams): the kernels' path choice
    restated on the host."""
    ids = np.asarray(ids, np.int64)
    items = sorted((s.start, s.stop, slot) for (b, s), slot in
                   ((it, block_to_slot[it[0]]) for it in layout))
    starts = np.array([i[0] for i in items], np.int64)
    ends = np.array([i[1] for i in items], np.int64)
    slots = np.array([i[2] for i in items], np.int64)
    pos = np.searchsorted(ends, ids, side="right")
    sr = slots[pos] * B + (ids - starts[pos])
    staged = ends_only = streamed = 0
    for c in range(ids.size // 32):
        i, s = ids[32 * c: 32 * c + 32], sr[32 * c: 32 * c + 32]
        lane = np.arange(32)
        ok = bool(np.all(i == i[0] + lane) and np.all(s == s[0] + lane))
        staged += ok
        streamed += ok and i[0] % 4 == 0
        ends_only += bool(i[31] == i[0] + 31 and s[31] == s[0] + 31)
    return staged, ends_only, streamed


def _layout(blocks, B, tail_block=None, tail_rows=None):
    """Packed slices in the listed order; `tail_block` gets `tail_rows` rows."""
    out, off = [], 0
    for b in blocks:
        n = tail_rows if b == tail_block else B
        out.append((int(b), slice(off, off + n)))
        off += n
    return out, off


def _whole_block_ids(layout, rng, frac=0.5, runs=3):
    """All rows of a few random runs of consecutive positions (~frac of them)."""
    npos = len(layout)
    take = np.zeros(npos, bool)
    span = max(1, int(frac * npos / runs))
    for _ in range(runs):
        s = int(rng.integers(0, npos))
        take[s:s + span] = True
    rows = [np.arange(sl.start, sl.stop) for (_, sl), t in zip(layout, take) if t]
    return np.concatenate(rows).astype(np.int64)


def _random_grads(rng, n):
    return {k: (rng.standard_normal((n, w)) * 1e-3).astype(np.float32) for k, w in WIDTHS.items()}


def _check_state(opt, oracle, layout, B):
    for b, sl in layout:
        rows = sl.stop - sl.start
        m, v = opt.export_block_state(b, rows=rows)
        slot = oracle._block_to_slot[b]
        for n in NAMES:
            np.testing.assert_array_equal(m[n].cpu().numpy(),
                                          oracle.exp_avg[n][slot * B: slot * B + rows],
                                          err_msg=f"m block {b} {n}")
            np.testing.assert_array_equal(v[n].cpu().numpy(),
                                          oracle.exp_avg_sq[n][slot * B: slot * B + rows],
                                          err_msg=f"v block {b} {n}")


# Each case: block size, the order in which the admitted blocks occupy the
# working set's positions (blocks are admitted in ascending id into the
# lowest free slots, so block k first holds slot k), an optional short tail
# block, and the minimum number of staged chunks the first step must contain.
CASES = {
    # 4-row blocks in slot order 0,5,2,3,4,1,6,7 (repeated): ids consecutive,
    # state rows not; the first and last rows of a 32-row chunk line up.
    "b4_permuted_slots": dict(B=4, order=[0, 5, 2, 3, 4, 1, 6, 7] + list(range(8, 64)),
                              tail=None, min_staged=1, misrouted=True),
    # 48-row blocks: chunks cross into the next position's slot; positions
    # 6 and 7 swapped so some crossings go to a non-adjacent slot.
    "b48_crossing": dict(B=48, order=[0, 1, 2, 3, 4, 5, 7, 6] + list(range(8, 40)),
                         tail=None, min_staged=20, misrouted=False),
    # 64-row blocks with a 50-row tail block (block 9) in the middle.
    "b64_tail_mid": dict(B=64, order=list(range(40)), tail=(9, 50), min_staged=20,
                         misrouted=False),
    # larger blocks, slots in reverse position order
    "b512_reversed": dict(B=512, order=list(range(23, -1, -1)), tail=(3, 300),
                          min_staged=100, misrouted=False),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_staged_whole_blocks_bit_exact_with_oracle(case):
    from tidegs_b200 import GPUResidentAdam

    cfg = CASES[case]
    B = cfg["B"]
    rng = np.random.default_rng(zlib.crc32(case.encode()))
    blocks = sorted(cfg["order"])
    tail_block, tail_rows = cfg["tail"] if cfg["tail"] else (None, None)
    layout, rows = _layout(cfg["order"], B, tail_block, tail_rows)
    params = {n: rng.standard_normal((rows, w)).astype(np.float32) for n, w in WIDTHS.items()}
    manager = _Manager(layout)
    g = _gaussians(manager, params)
    ref = {n: v.copy() for n, v in params.items()}
    opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=len(blocks), device="cuda")
    oracle = ResidentAdamOracle(batch_size=16, block_size=B, capacity_blocks=len(blocks))
    opt.set_resident_blocks(blocks)
    oracle.set_resident_blocks(blocks)

    for step in range(4):
        if step == 0:
            # every row of every block: all chunks that can stage do
            ids = np.concatenate([np.arange(s.start, s.stop) for _, s in layout]).astype(np.int64)
            ids.sort()
        elif step == 3:
            # whole blocks mixed with a sparse block in one launch
            ids = _whole_block_ids(layout, rng)
            b, sl = layout[len(layout) // 2]
            extra = np.arange(sl.start, sl.stop)[rng.random(sl.stop - sl.start) < 0.4]
            ids = np.unique(np.concatenate([ids, extra])).astype(np.int64)
        else:
            ids = _whole_block_ids(layout, rng)
        staged, ends_only, streamed = _staged_chunks(ids, layout, opt._block_to_slot, B)
        if step == 0:
            assert staged >= cfg["min_staged"], (staged, ends_only)
            assert streamed >= 1, "case must drive the bulk-copy pipeline"
            if cfg["misrouted"]:
                assert ends_only > staged, "case must contain a chunk whose ends alone line up"
        grads = _random_grads(rng, ids.size)
        s = opt.step(step + 1, g, torch.as_tensor(ids).cuda(),
                     {n: torch.as_tensor(x).cuda() for n, x in grads.items()})
        o = oracle.step(ref, ids, grads, layout, LRS, BETAS, EPS)
        assert s == o
        got = _values(g)
        for n in NAMES:
            np.testing.assert_array_equal(got[n], ref[n], err_msg=f"{case} step {step} {n}")
        _check_state(opt, oracle, layout, B)
        if step == 1:
            # Evict three blocks, then re-admit two of them together with a new
            # block: the re-admitted blocks and the newcomer sit in slots whose
            # rows still hold the evicted blocks' moments under an old stamp.
            gone = [blocks[1], blocks[len(blocks) // 2], blocks[-1]]
            keep = [b for b in blocks if b not in gone]
            opt.set_resident_blocks(keep)
            oracle.set_resident_blocks(keep)
            newcomer = max(blocks) + 1
            blocks = sorted(keep + gone[:2] + [newcomer])
            opt.set_resident_blocks(blocks)
            oracle.set_resident_blocks(blocks)
            # the newcomer takes the dropped block's position in the working set
            order = [newcomer if b == gone[2] else b for b, _ in layout]
            layout = [(b, sl) for b, (_, sl) in zip(order, layout)]
            manager.set_layout(layout)
    stats = opt.get_stats()
    for k in ("cold_restarts", "state_evictions"):
        assert stats[k] == oracle.stats[k], k


def test_full_size_whole_block_runs_sampled_bit_exact():
    """configs[3] shape: 2048 resident blocks x 16,384 rows, every row of the
    visible blocks (contiguous runs of blocks, ~30 % of them) updated, two
    steps, as the benchmark updates them: all chunks staged. The update of a
    row depends only on its own values and its slot's tables, so the oracle
    replaying 12 sampled visible blocks alone must match the full-size GPU
    result on them bit for bit."""
    from tidegs_b200 import GPUResidentAdam

    B, nb = 16384, 2048
    rows = B * nb
    rng = np.random.default_rng(23)
    order = rng.permutation(nb * 4)[:nb].tolist()
    layout = [(int(b), slice(i * B, (i + 1) * B)) for i, b in enumerate(order)]
    gen = torch.Generator(device="cuda").manual_seed(23)
    manager = _Manager(layout)
    g = types.SimpleNamespace(
        gpu_working_set_manager=manager,
        optimizer=types.SimpleNamespace(columns_lr=torch.tensor(LRS, dtype=torch.float32),
                                        param_groups=[{"betas": BETAS, "eps": EPS}]))
    for n in NAMES:
        setattr(g, ATTRS[n], torch.nn.Parameter(
            torch.randn((rows, WIDTHS[n]), generator=gen, device="cuda")))
    # visible positions: 16 runs of 24-56 consecutive positions
    vis = np.zeros(nb, bool)
    for _ in range(16):
        s = int(rng.integers(0, nb))
        vis[s:s + int(rng.integers(24, 57))] = True
    vis_pos = np.nonzero(vis)[0]
    sample = np.sort(rng.choice(vis_pos, 12, replace=False))
    sub_rows = torch.as_tensor(np.concatenate([np.arange(k * B, (k + 1) * B) for k in sample]),
                               device="cuda")
    ref = {n: getattr(g, ATTRS[n]).detach()[sub_rows].cpu().numpy() for n in NAMES}
    sub_layout = [(order[k], slice(i * B, (i + 1) * B)) for i, k in enumerate(sample)]
    opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=nb, device="cuda")
    oracle = ResidentAdamOracle(batch_size=16, block_size=B, capacity_blocks=len(sample))
    opt.set_resident_blocks([b for b, _ in layout])
    oracle.set_resident_blocks([b for b, _ in sub_layout])
    ids = (torch.as_tensor(vis_pos, device="cuda")[:, None] * B
           + torch.arange(B, device="cuda")[None, :]).reshape(-1)
    pick = torch.as_tensor(np.searchsorted(vis_pos, sample), device="cuda")
    for step in range(2):
        grads = {n: torch.randn((ids.numel(), w), generator=gen, device="cuda") * 1e-3
                 for n, w in WIDTHS.items()}
        stats = opt.step(step + 1, g, ids, grads)
        assert stats["touched_rows"] == ids.numel()
        assert stats["updated_blocks"] == vis_pos.size
        sub_ids = np.arange(len(sample) * B, dtype=np.int64)
        sel = (pick[:, None] * B + torch.arange(B, device="cuda")[None, :]).reshape(-1)
        sub_grads = {n: x[sel].cpu().numpy() for n, x in grads.items()}
        oracle.step(ref, sub_ids, sub_grads, sub_layout, LRS, BETAS, EPS)
        for n in NAMES:
            got = getattr(g, ATTRS[n]).detach()[sub_rows].cpu().numpy()
            np.testing.assert_array_equal(got, ref[n], err_msg=f"{n} step {step}")
        for i, k in enumerate(sample[:3]):
            m, v = opt.export_block_state(order[k])
            slot = oracle._block_to_slot[order[k]]
            for n in NAMES:
                np.testing.assert_array_equal(m[n].cpu().numpy(),
                                              oracle.exp_avg[n][slot * B:(slot + 1) * B])
                np.testing.assert_array_equal(v[n].cpu().numpy(),
                                              oracle.exp_avg_sq[n][slot * B:(slot + 1) * B])
        del grads


# ---------------------------------------------------------------------------
# Pull kernel (multi-GPU owner update, ranks emulated on one GPU)
# ---------------------------------------------------------------------------
def _rank_block_tile(rank, block, B):
    r = np.random.default_rng(7919 * rank + int(block))
    return (r.standard_normal((B, 59)) * 1e-3).astype(np.float32)


def _rank_grads(rank, blocks, B):
    """SoA gradients of a rank: its rendered blocks in ascending id, B rows each."""
    aos = (np.concatenate([_rank_block_tile(rank, b, B) for b in blocks]) if len(blocks)
           else np.zeros((0, 59), np.float32))
    return {n: torch.from_numpy(aos[:, ob.UNIFIED[n]:ob.UNIFIED[n] + w].copy()).cuda()
            for n, w in ob.WIDTHS.items()}


def _rank_order_sum(vis, block, B):
    """Contributions of `block` summed in rank order, one rounding per addition."""
    s = None
    for r, v in enumerate(vis):
        if block in v:
            t = _rank_block_tile(r, block, B)
            s = t.copy() if s is None else (s + t).astype(np.float32)
    return s


@pytest.mark.parametrize("W,B,reorder,ctas", [(3, 64, False, 0), (2, 32, True, 0),
                                              (4, 96, True, 0), (2, 48, False, 0),
                                              (3, 2048, True, 0), (3, 2048, False, 5)])
def test_pull_staged_bit_exact_with_oracle(W, B, reorder, ctas):
    """The owner's pull update over whole exchanged blocks equals the oracle
    update on the rank-order sum of the senders' gradients, bit for bit;
    three steps with an eviction and re-admission before the last one.
    `reorder` puts the owned blocks in the working set in an order unlike
    their slot order; `ctas` caps the streamed kernel's grid (0: one CTA per
    SM), so that few CTAs walk many chunks each."""
    from tidegs_b200 import GPUResidentAdam
    from tidegs_b200.sharded import PeerGradPull, make_plan

    rng = np.random.default_rng(100 + W * 7 + B)
    nb = 60 if B <= 96 else 16
    vis = [sorted(set(rng.integers(0, nb, nb // 2).tolist())) for _ in range(W)]
    owner = W - 1
    blocks_all = sorted(set(b for v in vis for b in v if b % W == owner))
    order = list(reversed(blocks_all)) if reorder else list(blocks_all)
    out_order = {b: i for i, b in enumerate(order)}
    plan = make_plan(vis, W, owner, B, out_order=out_order)
    owned = plan.out_blocks.tolist()
    assert owned == order
    grads = [_rank_grads(r, sorted(int(b) for b in make_plan(vis, W, r, B).send_blocks), B)
             for r in range(W)]
    rows = len(owned) * B
    layout = [(b, slice(i * B, (i + 1) * B)) for i, b in enumerate(owned)]
    params = {n: rng.standard_normal((rows, w)).astype(np.float32) for n, w in WIDTHS.items()}
    manager = _Manager(layout)
    g = _gaussians(manager, params)
    ref = {n: v.copy() for n, v in params.items()}
    opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=len(owned), device="cuda")
    oracle = ResidentAdamOracle(batch_size=16, block_size=B, capacity_blocks=len(owned))
    opt.set_resident_blocks(owned)
    oracle.set_resident_blocks(owned)
    pull = PeerGradPull.in_process(grads, owner, B, "cuda")
    pull.max_ctas = ctas
    ids = np.arange(rows, dtype=np.int64)
    summed = np.concatenate([_rank_order_sum(vis, b, B) for b in owned])
    ref_grads = {n: summed[:, ob.UNIFIED[n]:ob.UNIFIED[n] + w].copy() for n, w in ob.WIDTHS.items()}
    if B % 32 == 0:
        staged, _, streamed = _staged_chunks(ids, layout, opt._block_to_slot, B)
        assert staged == streamed == rows // 32
    for step in range(3):
        s = opt.step_pulled(step + 1, g, torch.as_tensor(ids).cuda(), pull, plan)
        o = oracle.step(ref, ids, ref_grads, layout, LRS, BETAS, EPS)
        assert s == o
        got = _values(g)
        for n in NAMES:
            np.testing.assert_array_equal(got[n], ref[n], err_msg=f"W={W} B={B} step {step} {n}")
        _check_state(opt, oracle, layout, B)
        if step == 1:
            # evict two owned blocks and re-admit them: new stamps, stale rows
            gone = owned[:1] + owned[-1:]
            keep = [b for b in owned if b not in gone]
            opt.set_resident_blocks(keep)
            oracle.set_resident_blocks(keep)
            opt.set_resident_blocks(owned)
            oracle.set_resident_blocks(owned)
    assert opt.get_stats()["cold_restarts"] == oracle.stats["cold_restarts"]
