"""Benchmark of the tidegs_b200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tidegs_b200|reference]

Workload (the largest single-GPU configuration; under
torchrun each rank runs it on its own blocks, rank = block_id mod world):
one "step" = one iteration of the resident-block path over 2048 slots x 16,384
Gaussians x 59 fp32 (33.5 M Gaussians per GPU):
  1. fused resident Adam over the rows of the visible blocks (camera batch of
     16 contiguous block runs, ~30 % of the slots),
  2. dirty marking of the updated blocks and their xyz bounds,
  3. dirty-and-evicted compaction of 512 evicted blocks (25 % turnover) and
     the CACHE-layout write-back pack of the dirty ones,
  4. materialization of 512 incoming blocks into the freed slots (packed rows
     -> component arrays + global ids, then the slot remap). The unpack into
     the loading buffer is enqueued before the pack: it does not depend on the
     write-back, and it keeps the device busy while the host waits for the
     dirty list.
`value` runs the step through the library entry points with every input
already in HBM; `e2e` runs it through the Python drop-in classes with the
incoming blocks streamed from a page-locked host pool (H2D inside the timed
region) and the write-back payload read back to host memory (D2H).
Metric: Gaussian parameter updates per second (Adam rows updated / s).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "Gaussian param-updates/sec per GPU & box (1/2/4/8 B200); HBM GB/s vs peak"
UNIT = "Gaussian updates/s"
B = 16384
SLOTS = 2048
TURNOVER = 512


# scene blocks a rank owns = POOL_MULT * SLOTS (4: BASELINE configs[3]'s
# pinned pool); lowered by plan_host_pool when the box's memory cannot hold
# every rank's page-locked host tier
POOL_MULT = 4
BLOCK_BYTES = B * 59 * 4


def set_slots(slots: int) -> None:
    """Resident slots per GPU; the turnover stays at 25 % of them."""
    global SLOTS, TURNOVER
    SLOTS = int(slots)
    TURNOVER = max(1, SLOTS // 4)


def host_memory_limit() -> int:
    """Bytes of host memory the job may use: MemTotal, or the cgroup limit
    when that is lower (the same value on every rank of the box)."""
    limit = None
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    limit = int(line.split()[1]) * 1024
                    break
    except OSError:
        pass
    for path in ("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory/memory.limit_in_bytes"):
        try:
            with open(path) as f:
                v = f.read().strip()
        except OSError:
            continue
        if v.isdigit() and int(v) > 0:
            limit = int(v) if limit is None else min(limit, int(v))
    return limit if limit is not None else 0


def plan_host_pool(world: int, host_tier: str, pool_blocks: int, limit: int):
    """(pool multiple, host tier) that fit every rank's host tier into 60 %
    of the box's memory: the cache holds POOL_MULT * SLOTS + TURNOVER
    page-locked entries plus pool_blocks seeded source blocks per rank; the
    scene shrinks to 3 or 2 x SLOTS blocks per rank before the cache gives
    way to the small fixed pool (pool_blocks page-locked blocks)."""
    budget = 0.6 * limit / world
    if host_tier == "cache":
        for mult in (4, 3, 2):
            if (mult * SLOTS + TURNOVER + pool_blocks) * BLOCK_BYTES <= budget:
                return mult, "cache"
        return 4, "pool"
    return 4, host_tier


WORKLOAD_CONFIG = {
    "workload": "configs[3]: full resident-set step, 2048 slots x 16384 Gaussians per GPU, "
                "16-camera contiguous block runs (~30% visible), 25% slot turnover, "
                "Bernoulli(0.5) dirty evictions"}

WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}
NAMES = tuple(WIDTHS)
ADAM_BYTES_PER_ROW = 59 * 4 * 7          # grad r + param r/w + m r/w + v r/w
# DRAM bytes per updated row of resident_adam_kernel measured by ncu:
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the 256-slot
# step (every input larger than L2) = 1654.8 MB over its 983,040 rows
ADAM_TRAFFIC_BYTES_PER_ROW = 1683.3
LRS = {"xyz": 1.6e-4, "opacity": 0.05, "scaling": 5e-3, "rotation": 1e-3, "features_dc": 2.5e-3,
       "features_rest": 1.25e-4}


# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        # the only collectives are one-element barriers and set-up gathers:
        # no use for NVLink multicast (NVLS) buffers
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.path = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", uuid], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.proc is None:
            return out
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return out
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        out["sm_mhz"] = statistics.median(sm) if sm else None
        out["sm_max_mhz"] = max(mx) if mx else None
        out["reasons"] = reasons
        out["samples"] = len(rows)
        return out


def measured_peak():
    path = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# Workload generation (seeded; shapes/distributions of BASELINE configs[3])
# ---------------------------------------------------------------------------
class Schedule:
    """Block ids, camera visibility and slot turnover for one rank."""

    def __init__(self, rank: int, world: int, seed: int = 4, n_cameras_sets: int = 4):
        self.rng = np.random.default_rng(seed + 1000 * rank)
        self.world = world
        self.rank = rank
        # owned block ids: rank + k*world; POOL_MULT * SLOTS per rank
        self.pool_ids = np.arange(rank, rank + world * POOL_MULT * SLOTS, world, dtype=np.int64)
        self.slot_block = self.rng.choice(self.pool_ids, SLOTS, replace=False)
        self.n_sets = n_cameras_sets

    _vis_cache: dict = {}

    def visible_positions(self, step: int) -> np.ndarray:
        """Union over 16 cameras of contiguous runs of slots, ~30 % visible
        (the same runs for every owner; cached per camera set)."""
        key = (SLOTS, step % self.n_sets)
        hit = Schedule._vis_cache.get(key)
        if hit is not None:
            return hit
        rng = np.random.default_rng(10_000 + step % self.n_sets)
        vis = np.zeros(SLOTS, bool)
        scale = SLOTS / 2048.0
        for _ in range(16):
            length = max(1, int(rng.integers(24, 56) * scale))
            start = int(rng.integers(0, max(1, SLOTS - length)))
            vis[start:start + length] = True
        out = np.nonzero(vis)[0]
        out.setflags(write=False)
        Schedule._vis_cache[key] = out
        return out

    def turnover(self, step: int):
        rng = np.random.default_rng(20_000 + step)
        evict_pos = np.sort(rng.choice(SLOTS, TURNOVER, replace=False))
        # pool blocks not resident, ascending (pool_ids is ascending)
        resident = np.zeros(self.pool_ids.size, bool)
        resident[(self.slot_block - self.rank) // self.world] = True
        candidates = self.pool_ids[~resident]
        incoming = np.sort(rng.choice(candidates, TURNOVER, replace=False))
        dirty = rng.random(TURNOVER) < 0.5
        return evict_pos, incoming, dirty

    def slot_table(self) -> np.ndarray:
        """Dense block id -> slot position table (-1: not resident)."""
        table = np.full(int(self.pool_ids[-1]) + 1, -1, np.int64)
        table[self.slot_block] = np.arange(SLOTS, dtype=np.int64)
        return table


def fill_params(comps, gen):
    rows = comps["xyz"].shape[0]
    comps["xyz"].uniform_(-100.0, 100.0, generator=gen)
    comps["features_dc"].normal_(0.0, 0.3, generator=gen)
    comps["features_rest"].normal_(0.0, 0.01, generator=gen)
    comps["opacity"].normal_(-2.0, 1.0, generator=gen)
    comps["scaling"].normal_(-4.0, 0.5, generator=gen)
    comps["rotation"].normal_(0.0, 1.0, generator=gen)
    comps["rotation"].div_(comps["rotation"].norm(dim=1, keepdim=True))
    assert rows > 0


# ---------------------------------------------------------------------------
# Device leg: library entry points, inputs resident in HBM
# ---------------------------------------------------------------------------
def rank_visible_positions(sched: "Schedule", step: int, world: int, rank: int) -> np.ndarray:
    """Slot positions of `sched`'s owner whose blocks rank `rank` renders at
    `step`: the owner's visible runs (~30 % of its slots, as on one GPU) split
    into `world` contiguous parts, each widened by 15 % of a part on both
    sides so that neighbouring ranks' cameras overlap."""
    pos = sched.visible_positions(step)
    if world == 1:
        return pos
    part = -(-pos.size // world)
    margin = int(0.15 * part)
    lo = max(0, rank * part - margin)
    hi = min(pos.size, (rank + 1) * part + margin)
    return pos[lo:hi]


def rendered_blocks(scheds, step: int, world: int):
    """Block ids whose gradients each rank renders at `step` (every owner's
    share for that rank)."""
    return [np.concatenate([o.slot_block[rank_visible_positions(o, step, world, r)]
                            for o in scheds]) for r in range(world)]


def exchange_capacity(sched: "Schedule", scheds, world: int):
    """(blocks a rank renders, tiles an owner receives): the largest over the
    periodic camera sets."""
    send_max = recv_max = 0
    for s_ in range(sched.n_sets):
        mine = sum(rank_visible_positions(o, s_, world, sched.rank).size for o in scheds)
        theirs = sum(rank_visible_positions(sched, s_, world, r).size for r in range(world))
        send_max, recv_max = max(send_max, mine), max(recv_max, theirs)
    return send_max, recv_max


class ScheduleTrace:
    """Every owner's synthetic schedule simulated ahead of the timed region
    (workload generation, not the measured path): for step k, the blocks
    each rank renders (vis[k], world > 1) and this rank's slot turnover
    (turn[k] = evicted slot positions, incoming block ids, dirty pattern)."""

    def __init__(self, world: int, rank: int, n_steps: int):
        scheds = [Schedule(o, world) for o in range(world)]
        self.vis, self.turn = [], []
        for k in range(n_steps):
            self.vis.append(rendered_blocks(scheds, k, world) if world > 1 else None)
            turns = [o.turnover(k) for o in scheds]
            self.turn.append(turns[rank])
            for o, (ev, inc, _) in zip(scheds, turns):
                o.slot_block[ev] = inc


class DeviceStep:
    def __init__(self, device, sched: Schedule, trace: ScheduleTrace, scheds=None, world: int = 1,
                 exchange: str = "pull"):
        from tidegs_b200 import _lib, _ops

        self._lib, self._ops = _lib, _ops
        self.device = device
        self.sched = sched
        self.trace = trace
        self.world = world
        self.scheds = scheds if scheds is not None else [sched]
        gen = torch.Generator(device=device).manual_seed(1234 + sched.rank)
        rows = SLOTS * B
        self.arena = {n: torch.empty((rows, w), device=device) for n, w in WIDTHS.items()}
        fill_params(self.arena, gen)
        self.gids = torch.empty(rows, dtype=torch.int64, device=device)
        _ops.fill_global_ids(self.gids, 0, _ops.i64_to_device(sched.slot_block, device), rows, B)
        # incoming blocks already landed in HBM (packed CACHE rows), 2 rotating sets
        self.incoming_pool = torch.empty((2 * TURNOVER * B, 59), device=device)
        self.incoming_pool.normal_(0.0, 1.0, generator=gen)
        self.loading = {n: torch.empty((TURNOVER * B, w), device=device) for n, w in WIDTHS.items()}
        self.loading_gids = torch.empty(TURNOVER * B, dtype=torch.int64, device=device)
        self.wb_staging = torch.empty((TURNOVER * B, 59), device=device)
        self.bounds = torch.empty((SLOTS, 6), device=device)
        # resident Adam state
        self.state = torch.zeros((rows, 128), device=device)
        self.slot_step = torch.zeros(SLOTS, dtype=torch.int32, device=device)
        self.stamp_host = np.ones(SLOTS, np.uint32)
        self.slot_stamp = torch.ones(SLOTS, dtype=torch.int32, device=device)
        self.slot_bias = torch.ones((SLOTS, 2), device=device)
        table = [(0.0, 0.0)] + [(float(np.float32(1 - 0.9 ** t)),
                                 float(np.float32(math.sqrt(1 - 0.999 ** t))))
                                for t in range(1, 20000)]
        self.table = torch.tensor(table, dtype=torch.float32, device=device)
        self.err = torch.zeros(4, dtype=torch.int32, device=device)
        self.pos_count = torch.zeros(SLOTS, dtype=torch.int32, device=device)
        starts = np.arange(SLOTS, dtype=np.int64) * B
        self.pos_start = _ops.i64_to_device(starts, device)
        self.pos_end = _ops.i64_to_device(starts + B, device)
        self.pos_slot = torch.arange(SLOTS, dtype=torch.int32, device=device)
        self.bitmap = torch.zeros(_ops.bitmap_words(int(sched.pool_ids.max()) + 1),
                                  dtype=torch.int32, device=device)
        # visible rows per camera set (all rows of visible blocks), grads
        self.vis_sets = []
        max_rows = 0
        for s in range(sched.n_sets):
            pos = sched.visible_positions(s)
            ids = (pos[:, None] * B + np.arange(B)[None, :]).reshape(-1)
            self.vis_sets.append((pos, _ops.i64_to_device(ids, device)))
            max_rows = max(max_rows, ids.size)
        self.grads = {n: torch.empty((max_rows, w), device=device).normal_(0, 1e-3, generator=gen)
                      for n, w in WIDTHS.items()}
        self.exchange_mode = exchange if world > 1 else None
        self.peer = None
        self.pull = None
        self.plan = None
        if world > 1:
            # gradients this rank renders for blocks of every owner, and the
            # exchange buffers (sizes: the largest of the periodic camera sets)
            send_max, recv_max = exchange_capacity(sched, self.scheds, world)
            self.rank_grads = {n: torch.empty((send_max * B, w), device=device).normal_(
                0, 1e-3, generator=gen) for n, w in WIDTHS.items()}
            if exchange == "pull":
                from tidegs_b200.sharded import PeerGradPull

                self.pull = PeerGradPull(self.rank_grads, B, device)
            elif exchange == "push":
                from tidegs_b200.sharded import PeerGradExchange

                self.peer = PeerGradExchange(B, capacity_blocks=recv_max, device=device)
            else:
                from tidegs_b200.sharded import BlockGradExchange

                self.exchange = BlockGradExchange(B, device=device)
                self.send_buf = torch.empty((send_max * B, 59), device=device)
                self.recv_buf = torch.empty((recv_max * B, 59), device=device)
            self.exchange_rows = 0
        self.adam_ms = []
        self.updated_rows = []
        torch.cuda.synchronize()

    def exchange_grads(self, k: int):
        """Owner-sharded gradient exchange of step k (world > 1): returns the
        owner's visible slot positions and local row ids; the reduced
        gradients land in self.grads."""
        W, me = self.world, self.sched.rank
        vis = self.trace.vis[k]
        if self._ahead is not None and self._ahead[0] == k:
            _, plan, slot_of, self.pull_tables = self._ahead  # built during step k-1
        else:
            plan, slot_of, self.pull_tables = self._make_plan(k, self.sched.slot_block)
        self._ahead = None
        # the rank's rendered gradients: its blocks in ascending id, B rows each
        starts = np.searchsorted(np.unique(vis[me]), plan.send_blocks).astype(np.int64) * B
        self._phase("plan")
        if self.pull is not None:
            # the owner's update kernel sums the senders' gradients itself
            self.plan = plan
            self.exchange_rows += int(plan.send_blocks.size) * B
        elif self.peer is not None:
            self.exchange_rows += self.peer.push(plan, self.rank_grads, starts, parity=k)
            self._phase("push")
            self.peer.barrier()
            self._phase("barrier")
            self.peer.reduce(plan, parity=k, out=self.grads, err=self.err)
            self._phase("owner_sum")
        else:
            send = self.exchange.pack(plan, self.rank_grads, starts, out=self.send_buf)
            recv = self.exchange.all_to_all(plan, send, out=self.recv_buf)
            self.exchange.reduce(plan, recv, out=self.grads, err=self.err)
            self.exchange_rows += int(send.shape[0])
        pos = slot_of[plan.out_blocks]
        # the owner's visible slots are its camera set's positions: reuse the
        # device row ids prepared for that set
        set_pos, set_ids = self.vis_sets[k % self.sched.n_sets]
        if not np.array_equal(pos, set_pos):
            raise RuntimeError("exchange plan and owner visibility disagree")
        return pos, set_ids

    def _make_plan(self, k: int, slot_block: np.ndarray):
        """Exchange plan of step k for the slot map `slot_block` (and, for the
        pull exchange, its device tables)."""
        from tidegs_b200.sharded import make_plan

        table = np.full(int(self.sched.pool_ids[-1]) + 1, -1, np.int64)
        table[slot_block] = np.arange(slot_block.size, dtype=np.int64)
        plan = make_plan(self.trace.vis[k], self.world, self.sched.rank, B, out_order=table)
        tables = self.pull.tables(plan) if self.pull is not None else None
        return plan, table, tables

    def plan_ahead(self, k: int):
        """Builds step k+1's plan on the host while the GPU runs step k (the
        slot map after step k's turnover is known from the schedule)."""
        if self.world == 1 or k + 1 >= len(self.trace.turn):
            return
        ev, inc, _ = self.trace.turn[k]
        nxt = self.sched.slot_block.copy()
        nxt[ev] = inc
        self._ahead = (k + 1,) + self._make_plan(k + 1, nxt)

    _ahead = None
    pull_tables = None

    def adam(self, ids: torch.Tensor, timed: bool):
        _lib = self._lib
        n = ids.numel()
        stream = _lib.stream_handle(self.device)
        c = _lib.ResidentCountArgs(
            pos_start=self.pos_start.data_ptr(), pos_end=self.pos_end.data_ptr(),
            pos_slot=self.pos_slot.data_ptr(), n_positions=SLOTS, block_size=B,
            param_rows=SLOTS * B, local_ids=ids.data_ptr(), n_rows=n,
            slot_step=self.slot_step.data_ptr(), slot_stamp=self.slot_stamp.data_ptr(),
            slot_bias=self.slot_bias.data_ptr(), step_table=self.table.data_ptr(),
            step_table_len=self.table.shape[0], n_slots=SLOTS,
            pos_count=self.pos_count.data_ptr(), err=self.err.data_ptr())
        tables = self.pull_tables
        _lib.call("tgs_resident_adam_count", c, stream)
        self._phase("count")
        a = _lib.ResidentAdamArgs()
        for i, name in enumerate(NAMES):
            a.param[i] = self.arena[name].data_ptr()
            a.grad[i] = self.grads[name].data_ptr()
            a.lr[i] = LRS[name]
        a.beta1, a.beta2, a.eps = 0.9, 0.999, 1e-15
        a.one_minus_beta1, a.one_minus_beta2 = 1.0 - 0.9, 1.0 - 0.999
        a.batch_size = 16.0
        a.pos_start, a.pos_end, a.pos_slot = (self.pos_start.data_ptr(), self.pos_end.data_ptr(),
                                              self.pos_slot.data_ptr())
        a.n_positions, a.block_size = SLOTS, B
        a.local_ids, a.n_rows = ids.data_ptr(), n
        a.state, a.slot_stamp = self.state.data_ptr(), self.slot_stamp.data_ptr()
        a.slot_bias, a.err = self.slot_bias.data_ptr(), self.err.data_ptr()
        if self.pull is not None:
            self.pull.barrier()  # every rank's gradients of this step are written
            self._phase("acquire")
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        if self.pull is not None:
            self.pull.launch(a, self.plan, stream, tables=tables)
        else:
            _lib.call("tgs_resident_adam_apply", a, stream)
        if timed:
            e1.record()
            self.adam_ms.append((e0, e1, n))
        self._phase("adam")
        if self.pull is not None:
            self.pull.barrier()  # no owner still reads this step's gradients
            self._phase("release")

    phase_ms = None  # {phase: [ms, ...]} when per-phase timing is on
    host_ms = None   # host time between the same marks

    def _phase(self, name):
        if self.phase_ms is None:
            return
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self._events.append((name, ev, time.perf_counter()))

    def collect_phases(self):
        if self.phase_ms is None:
            return
        torch.cuda.synchronize()
        for (_, e0, h0), (name, e1, h1) in zip(self._events, self._events[1:]):
            self.phase_ms.setdefault(name, []).append(e0.elapsed_time(e1))
            self.host_ms.setdefault(name, []).append((h1 - h0) * 1e3)
        self._events = []

    def step(self, k: int, timed: bool = False) -> int:
        _ops = self._ops
        sched = self.sched
        self._events = []
        self._phase("start")
        if self.world > 1:
            # 0. gradients of blocks rendered on other ranks reach their owners
            pos, ids = self.exchange_grads(k)
            self._phase("exchange")
        else:
            pos, ids = self.vis_sets[k % sched.n_sets]
        # 1. optimizer over the visible rows
        self.adam(ids, timed)
        self.plan_ahead(k)
        # 2. updated blocks are dirty; refresh their bounds
        updated = sched.slot_block[pos]
        _ops.dirty_mark(self.bitmap, updated.tolist(), True)
        _ops.block_bounds(self.arena["xyz"], (pos * B).tolist(), [B] * pos.size,
                          self.bounds[: pos.size])
        self._phase("dirty_bounds")
        # 3. evict 512 slots: write back the dirty ones
        evict_pos, incoming, dirty = self.trace.turn[k]
        # half of the evicted blocks were never touched before: mark a random
        # dirty pattern so that the compaction has work of the configured mix
        evicted_blocks = sched.slot_block[evict_pos]
        _ops.dirty_mark(self.bitmap, evicted_blocks[dirty].tolist(), True)
        _ops.dirty_mark(self.bitmap, evicted_blocks[~dirty].tolist(), False)
        order = np.argsort(evicted_blocks, kind="stable")
        selection = _ops.dirty_select_async(self.bitmap, evicted_blocks[order].tolist())
        self._phase("dirty_select")
        # 4. materialize the incoming blocks into the loading buffer; this does
        # not depend on the write-back, so the device runs it while the host
        # waits for the dirty list and plans the pack
        src = self.incoming_pool[(k % 2) * TURNOVER * B:(k % 2 + 1) * TURNOVER * B]
        ids_dev = _ops.i64_to_device(incoming, self.device)
        _ops.unpack_rows(src, self._lib.LAYOUT_CACHE, self.loading, 0,
                         global_ids=self.loading_gids, block_ids=ids_dev, block_size=B)
        self._phase("unpack")
        wb_ids = selection.wait()
        sorted_blocks = evicted_blocks[order]
        wb_pos = evict_pos[order][np.searchsorted(sorted_blocks, np.asarray(wb_ids, np.int64))]
        _ops.pack_rows(self.arena, (wb_pos * B).tolist(), [B] * wb_pos.size,
                       self.wb_staging[: wb_pos.size * B], self._lib.LAYOUT_CACHE)
        self._phase("pack")
        _ops.dirty_mark(self.bitmap, wb_ids, False)
        self._phase("writeback")
        # 5. evicted slots take the incoming blocks
        _ops.copy_blocks(self.loading, self.loading_gids, self.arena, self.gids,
                         (np.arange(TURNOVER) * B).tolist(), (evict_pos * B).tolist(),
                         [B] * TURNOVER, self.device)
        self._phase("slot_copy")
        sched.slot_block[evict_pos] = incoming
        self.stamp_host[evict_pos] += 1
        _ops.upload_into(self.slot_stamp, self.stamp_host.view(np.int32))
        self.slot_step.index_fill_(0, _ops.i64_to_device(evict_pos, self.device), 0)
        self._phase("tables")
        return int(ids.numel())

    def close(self):
        """Releases the peer mappings (collective over the ranks)."""
        for attr in ("peer", "pull"):
            obj = getattr(self, attr)
            if obj is not None:
                obj.close()
                setattr(self, attr, None)

    def adam_stats(self):
        ms = [e0.elapsed_time(e1) for e0, e1, _ in self.adam_ms]
        rows = [n for _, _, n in self.adam_ms]
        return ms, rows


class _Skipped(Exception):
    pass


# ---------------------------------------------------------------------------
# e2e leg: Python drop-in classes, host pool -> HBM -> host
# ---------------------------------------------------------------------------
class _SceneStore:
    """Block store behind the e2e host tier: block b's rows are
    distinct[b % len(distinct)]; write_patch (the disk tier, not measured)
    only counts. Once sealed, a read means the host tier missed."""

    def __init__(self, distinct: torch.Tensor):
        self.distinct = distinct
        self.sealed = False
        self.patches = 0

    def read_blocks(self, block_ids):
        if self.sealed:
            raise RuntimeError(f"host tier miss for blocks {list(block_ids)[:8]}")
        n = self.distinct.shape[0]
        return {int(b): self.distinct[int(b) % n] for b in block_ids}

    def write_patch(self, blocks):
        self.patches += 1
        return self.patches


class ApiStep:
    """The step through the Python drop-ins. Slice position i of the active
    buffer holds sched.slot_block[i]; the persistent-slot plan gives incoming
    blocks (ascending) the freed slices (ascending), which is exactly the
    schedule's turnover, so every rank can replicate every owner's layout."""

    profile = None
    _pending_activate = False

    def _mark(self, name, t):
        if self.profile is not None:
            now = time.perf_counter()
            self.profile[name] = self.profile.get(name, 0.0) + now - t
            return now
        return t

    def __init__(self, device, scheds, trace: ScheduleTrace, rank: int, world: int,
                 pool_blocks: int, exchange: str = "pull", host_tier: str = "cache"):
        import types

        from tidegs_b200 import (BlockLayout, CachedBlockReader, DoubleBufferGPUWorkingSet,
                                 GPUResidentAdam, GPUWorkingSet, PinnedBlockCache,
                                 PinnedBlockPool, _ops)

        self.device = device
        self.scheds = scheds
        self.trace = trace
        self.sched = sched = scheds[rank]
        self.rank, self.world = rank, world
        num_total = int(max(int(o.pool_ids.max()) for o in scheds) + 1) * B
        gen = torch.Generator().manual_seed(99 + rank)
        self.cache = None
        if host_tier == "cache":
            # the host tier holds every scene block of this rank (POOL_MULT x
            # SLOTS blocks, BASELINE configs[3]'s pinned pool): pool_blocks distinct
            # seeded blocks, block b holding distinct[b % pool_blocks], read
            # into the cache's page-locked slab through its prefetch; room
            # for one write-back batch of fresh entries on top
            distinct = torch.empty((pool_blocks, B, 59))
            for i in range(pool_blocks):
                distinct[i].normal_(0.0, 1.0, generator=gen)
            store = _SceneStore(distinct)
            self.cache = PinnedBlockCache(store, max_ram_gb=1e9, block_size=B, verbose=False,
                                          capacity_blocks=sched.pool_ids.size + TURNOVER)
            self.cache.prefetch(sched.pool_ids.tolist())
            store.sealed = True  # a host-tier miss inside the steps is an error
            self.pool = CachedBlockReader(self.cache, num_total, B)
        else:
            data = torch.empty((pool_blocks, B, 59), pin_memory=True)
            for i in range(pool_blocks):
                data[i].normal_(0.0, 1.0, generator=gen)
            self.pool = PinnedBlockPool(data, B, num_total, layout=BlockLayout.CACHE)
        self.db = DoubleBufferGPUWorkingSet(num_total, B, device=device, verbose=False)
        self.ws = GPUWorkingSet(num_total, B, device=device)
        self.opt = GPUResidentAdam(batch_size=16, block_size=B, capacity_blocks=SLOTS,
                                   device=device)
        act = self.db.active_buffer
        order = [int(b) for b in sched.slot_block]
        self.db._allocate_target_tensors(act, SLOTS * B)
        fill_params(act.components(), torch.Generator(device=device).manual_seed(5))
        _ops.fill_global_ids(act.local_to_global_idx, 0, _ops.i64_to_device(order, device),
                             SLOTS * B, B)
        act.loaded_blocks = list(order)
        act.block_to_local_slice = {b: slice(i * B, (i + 1) * B) for i, b in enumerate(order)}
        act.num_gaussians = SLOTS * B
        self.gaussians = types.SimpleNamespace(
            gpu_working_set_manager=self.ws,
            optimizer=types.SimpleNamespace(
                columns_lr=torch.tensor([LRS[n] for n in NAMES], dtype=torch.float32),
                param_groups=[{"betas": (0.9, 0.999), "eps": 1e-15}]))
        self._activate()
        self.opt.set_resident_blocks(order)
        # visible rows of each camera set, page-locked (world == 1)
        self.ids_pinned = []
        for s_ in range(sched.n_sets):
            pos = sched.visible_positions(s_)
            self.ids_pinned.append(
                torch.from_numpy((pos[:, None] * B + np.arange(B)[None, :]).reshape(-1)).pin_memory())
        max_rows = max(t.numel() for t in self.ids_pinned)
        self.grads = {n: torch.empty((max_rows, w), device=device).normal_(0, 1e-3)
                      for n, w in WIDTHS.items()}
        self.peer = None
        self.pull = None
        if world > 1:
            send_max, recv_max = exchange_capacity(sched, scheds, world)
            self.rank_grads = {n: torch.empty((send_max * B, w), device=device).normal_(0, 1e-3)
                               for n, w in WIDTHS.items()}
            if exchange == "pull":
                from tidegs_b200.sharded import PeerGradPull

                self.pull = PeerGradPull(self.rank_grads, B, device)
            elif exchange == "push":
                from tidegs_b200.sharded import PeerGradExchange

                self.peer = PeerGradExchange(B, capacity_blocks=recv_max, device=device)
            else:
                from tidegs_b200.sharded import BlockGradExchange

                self.exchange = BlockGradExchange(B, device=device)
                self.send_buf = torch.empty((send_max * B, 59), device=device)
                self.recv_buf = torch.empty((recv_max * B, 59), device=device)
        # page-lock the write-back staging once, at its largest size (every
        # evicted block dirty), instead of growing it inside timed steps
        if self.cache is None:
            for _ in range(2):
                _, _, ready = self.ws._acquire_writeback_staging(TURNOVER * B)
                ready.set()
        else:
            self.ws.ensure_direct_writeback_capacity(TURNOVER * B)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        torch.cuda.synchronize()

    def _activate(self):
        act = self.db.active_buffer
        ws = self.ws
        ws.gpu_xyz, ws.gpu_scaling, ws.gpu_rotation = act.xyz, act.scaling, act.rotation
        ws.gpu_opacity, ws.gpu_features_dc = act.opacity, act.features_dc
        ws.gpu_features_rest = act.features_rest
        ws.local_to_global_idx = act.local_to_global_idx
        ws.loaded_blocks = list(act.loaded_blocks)
        ws.block_to_gpu_slice.clear()
        ws.block_to_gpu_slice.update(act.block_to_local_slice)
        g = self.gaussians
        g._xyz, g._opacity, g._scaling = act.xyz, act.opacity, act.scaling
        g._rotation, g._features_dc, g._features_rest = act.rotation, act.features_dc, act.features_rest

    def _grads_and_ids(self, k: int):
        """(sparse_grad_local_ids, sparse_grad_components or (pull, plan)) of
        this owner."""
        if self.world == 1:
            ids_host = self.ids_pinned[k % self.sched.n_sets]
            n = ids_host.numel()
            self.h2d_bytes += n * 8
            return self._upload_ids(ids_host), {name: g[:n] for name, g in self.grads.items()}
        from tidegs_b200.sharded import make_plan

        W, me = self.world, self.rank
        vis = self.trace.vis[k]
        # slice position i of the active buffer holds sched.slot_block[i]
        slot_of = self.sched.slot_table()
        plan = make_plan(vis, W, me, B, out_order=slot_of)
        starts = np.searchsorted(np.unique(vis[me]), plan.send_blocks).astype(np.int64) * B
        if self.pull is not None:
            grads = (self.pull, plan)
        elif self.peer is not None:
            self.peer.push(plan, self.rank_grads, starts, parity=k)
            self.peer.barrier()
            grads = self.peer.reduce(plan, parity=k, out=self.grads)
        else:
            send = self.exchange.pack(plan, self.rank_grads, starts, out=self.send_buf)
            recv = self.exchange.all_to_all(plan, send, out=self.recv_buf)
            grads = self.exchange.reduce(plan, recv, out=self.grads)
        rows = slot_of[plan.out_blocks] * B
        ids_host = self.ids_pinned[k % self.sched.n_sets]
        slices = self.db.active_buffer.block_to_local_slice
        probe = plan.out_blocks[:: max(1, plan.n_out // 16)]
        if (not np.array_equal(rows, ids_host[::B].numpy())
                or any(slices[int(b)].start != slot_of[int(b)] * B for b in probe)):
            raise RuntimeError("exchange plan and owner slices disagree")
        self.h2d_bytes += ids_host.numel() * 8
        return self._upload_ids(ids_host), grads

    def close(self):
        """Releases the peer mappings (collective over the ranks) and stops
        the host tier's workers."""
        for attr in ("peer", "pull"):
            obj = getattr(self, attr)
            if obj is not None:
                obj.close()
                setattr(self, attr, None)
        if self.cache is not None:
            self.cache.shutdown()

    def _upload_ids(self, ids_host: torch.Tensor) -> torch.Tensor:
        """Row ids from page-locked memory, read by a kernel (not queued
        behind the prefetch's block DMA on the copy engine)."""
        from tidegs_b200 import _lib

        out = torch.empty(ids_host.numel(), dtype=torch.int64, device=self.device)
        _lib.call("tgs_copy_small", out.data_ptr(), ids_host.data_ptr(), ids_host.numel() * 8,
                  torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def step(self, k: int) -> int:
        """One iteration in the engine's order: the resident plan for k+1 is
        known up front and its N+1 prefetch (H2D of the incoming blocks) runs
        on the worker thread / prefetch stream while the optimizer step and
        the write-back of iteration k run."""
        db, ws, sched = self.db, self.ws, self.sched
        t = time.perf_counter()
        if self.profile is not None:
            step_ev = torch.cuda.Event(enable_timing=True)
            step_ev.record()
            db.prefetch_events = {}
        evict_pos, incoming_arr, _ = self.trace.turn[k]
        evicted_arr = np.sort(sched.slot_block[evict_pos])
        evicted = evicted_arr.tolist()
        incoming = incoming_arr.tolist()
        keep = np.setdiff1d(sched.slot_block, evicted_arr, assume_unique=True).tolist()
        t = self._mark("plan", t)
        db.start_prefetch(iteration=k + 1, visible_block_ids=keep + incoming,
                          resident_block_ids=keep, evicted_block_ids=evicted,
                          block_reader=self.pool, defer_resident_copy=True)
        t = self._mark("start_prefetch", t)
        if self._pending_activate:
            # the views of the slots swapped in at the end of the previous
            # step (after the N+1 DMA is queued: it needs only the slot map)
            self._activate()
            self.opt.set_resident_blocks(db.active_buffer.loaded_blocks)
            self._pending_activate = False
            t = self._mark("activate", t)
        ids, grads = self._grads_and_ids(k)
        t = self._mark("exchange", t)
        if isinstance(grads, tuple):
            stats = self.opt.step_pulled(k, self.gaussians, ids, *grads)
        else:
            stats = self.opt.step(k, self.gaussians, ids, grads)
        t = self._mark("adam_step", t)
        updated = stats["updated_block_ids"]
        db.mark_dirty_blocks(updated)
        bounds = ws.stage_block_bounds(updated)
        t = self._mark("dirty_mark_bounds", t)
        wb_ids = db.dirty_blocks_for_eviction(evicted)
        t = self._mark("dirty_select", t)
        pending = ws.stage_updated_blocks(wb_ids, host_cache=self.cache)
        t = self._mark("stage_writeback", t)
        if pending is not None:
            payload = pending.wait()
            self.d2h_bytes += sum(v.numel() * 4 for v in payload.values())
            pending.release()
        t = self._mark("writeback_wait", t)
        db.mark_blocks_written_back(wb_ids)
        if bounds is not None:
            bounds.wait()
            self.d2h_bytes += bounds.cpu_bounds.numel() * 4
        db.finalize_retained_blocks(keep, target="loading")
        t = self._mark("bounds_finalize", t)
        db.wait_for_prefetch(k + 1)
        t = self._mark("wait_prefetch", t)
        if self.profile is not None:
            # device timeline of the N+1 prefetch, relative to the step start
            end_ev = torch.cuda.Event(enable_timing=True)
            end_ev.record()
            end_ev.synchronize()
            for name, ev in db.prefetch_events.items():
                key = "dev_" + name
                self.profile[key] = self.profile.get(key, 0.0) + step_ev.elapsed_time(ev) / 1e3
            key = "dev_wait_prefetch_done"
            self.profile[key] = self.profile.get(key, 0.0) + step_ev.elapsed_time(end_ev) / 1e3
            db.prefetch_events = None
            t = time.perf_counter()
        db.swap_buffers()
        t = self._mark("swap", t)
        sched.slot_block[evict_pos] = incoming_arr
        self._pending_activate = True
        self.h2d_bytes += TURNOVER * B * 59 * 4
        return int(ids.numel())


# ---------------------------------------------------------------------------
# Diagnostic: the pull kernel with a remote sender, in one process
# ---------------------------------------------------------------------------
def pull_probe(args, modes):
    """Not the bench line. One owner (GPU 0) of a two-rank schedule updates
    its visible rows with the pull kernel while the other rank's gradients
    live on GPU 1 ("remote", read over NVLink) or on GPU 0 ("local"), next to
    the single-GPU kernel ("plain"). One JSON line per mode (CUDA events)."""
    from tidegs_b200.sharded import PeerGradPull, make_plan

    W = 2
    torch.cuda.set_device(0)
    d0 = torch.device("cuda", 0)
    scheds = [Schedule(r, W) for r in range(W)]
    ds = DeviceStep(d0, scheds[0], None, scheds=scheds, world=1)
    caps = [exchange_capacity(scheds[r], scheds, W)[0] for r in range(W)]
    plan = make_plan(rendered_blocks(scheds, 0, W), W, 0, B, out_order=scheds[0].slot_table())
    pos, ids = ds.vis_sets[0]
    if not np.array_equal(scheds[0].slot_table()[plan.out_blocks], pos):
        raise RuntimeError("probe plan and owner visibility disagree")
    for mode in modes:
        ds.pull = ds.pull_tables = None
        if mode != "plain":
            where = [d0, torch.device("cuda", 1) if mode == "remote" else d0]
            grads = [{n: torch.empty((caps[r] * B, w), device=where[r]).normal_(0, 1e-3)
                      for n, w in WIDTHS.items()} for r in range(W)]
            ds.pull = PeerGradPull.in_process(grads, 0, B, d0)
            ds.plan, ds.pull_tables = plan, ds.pull.tables(plan)
        ds.adam_ms = []
        for k in range(args.warmup + args.steps):
            ds.adam(ids, timed=k >= args.warmup)
        torch.cuda.synchronize()
        ms = sorted(ms for ms, _ in zip(*ds.adam_stats()))
        print(json.dumps({"probe": mode, "rows": int(ids.numel()), "median_ms": ms[len(ms) // 2],
                          "contributions": int(plan.contrib_offsets[-1]), "blocks": plan.n_out,
                          "remote_blocks": int(sum(plan.recv_counts[1:]))}), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Diagnostic: touched-only gradient accumulation of a camera batch
# ---------------------------------------------------------------------------
def _look_at(eye, target, up=(0.0, 0.0, 1.0)) -> np.ndarray:
    """OpenGL view matrix (camera looks down -Z)."""
    eye, target, up = (np.asarray(v, dtype=np.float64) for v in (eye, target, up))
    f = (target - eye) / np.linalg.norm(target - eye)
    s = np.cross(f, up)
    s /= np.linalg.norm(s)
    m = np.eye(4)
    m[0, :3], m[1, :3], m[2, :3] = s, np.cross(s, f), -f
    m[:3, 3] = -m[:3, :3] @ eye
    return m


def _perspective(fovy_deg: float, aspect: float, near: float, far: float) -> np.ndarray:
    t = 1.0 / np.tan(np.radians(fovy_deg) / 2.0)
    m = np.zeros((4, 4))
    m[0, 0], m[1, 1] = t / aspect, t
    m[2, 2], m[2, 3] = (far + near) / (near - far), 2.0 * far * near / (near - far)
    m[3, 2] = -1.0
    return m


def cull_probe(args):
    """Not the bench line. Frustum culling of a configs[4]-sized scene
    (61,036 block spheres, blocks of 16,384 Gaussians in a 200^3 box) for a
    16-camera batch: BlockCuller (one launch; device time with CUDA events,
    and with the per-camera id lists read back to Python lists) against the
    reference's per-camera numpy evaluation (oracle/culling.py, the same
    numpy operations) on the host; checks the visible sets are equal."""
    import warnings

    from oracle import culling as oc
    from tidegs_b200 import BlockCuller

    warnings.filterwarnings("ignore", message="Suspicious plane orientations")
    torch.cuda.set_device(0)
    rng = np.random.default_rng(11)
    n = 61036
    centers = rng.uniform(-100.0, 100.0, (n, 3))
    half = rng.uniform(1.0, 6.0, (n, 3))
    bounds = np.concatenate([centers - half, centers + half], axis=1).astype(np.float32)
    cams = []
    for _ in range(16):
        ang = rng.uniform(0, 2 * np.pi)
        eye = np.array([110 * np.cos(ang), 110 * np.sin(ang), rng.uniform(10, 60)])
        cams.append((_look_at(eye, rng.uniform(-60, 60, 3)),
                     _perspective(rng.uniform(25, 45), 16 / 9, 0.5, 260.0)))
    from tidegs_b200.culling import extract_frustum_planes

    cu = BlockCuller(torch.from_numpy(bounds).cuda(), verbose=False)
    planes_ms, dev_ms, list_ms = [], [], []
    for k in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        planes = np.stack([extract_frustum_planes(v, p) for v, p in cams])
        t1 = time.perf_counter()
        cu.cull_cameras(None, planes=planes, as_tensors=True)  # uploads stay out of the timing
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ids, counts = cu.cull_cameras(None, planes=planes, as_tensors=True)
        e1.record()
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        lists = cu.cull_cameras(cams)
        t3 = time.perf_counter()
        if k >= args.warmup:
            planes_ms.append((t1 - t0) * 1e3)
            dev_ms.append(e0.elapsed_time(e1))
            list_ms.append((t3 - t2) * 1e3)
    c_np, r_np = oc.spheres(bounds)
    t0 = time.perf_counter()
    want = [oc.visible(c_np, r_np, oc.planes(v, p)).tolist() for v, p in cams]
    cpu_ms = (time.perf_counter() - t0) * 1e3
    if want != lists:
        raise RuntimeError("cull-probe: visible sets differ from the oracle")
    vis = sum(len(x) for x in want)
    print(json.dumps({"probe": "frustum_cull", "blocks": n, "cameras": 16,
                      "visible_fraction": round(vis / (16 * n), 3),
                      "host_planes_ms": round(statistics.median(planes_ms), 3),
                      "gpu_launch_ms": round(statistics.median(dev_ms), 4),
                      "gpu_with_python_lists_ms": round(statistics.median(list_ms), 3),
                      "reference_numpy_ms": round(cpu_ms, 2), "equal": True}), flush=True)


def render_probe(args):
    """Not the bench line. The engine's render path for one camera batch
    (strategies/tide_engine/engine.py:481-561): projection, tile intersection,
    SH colors (degree 3), rasterization forward and the three backward
    kernels, tidegs_b200 against
    the reference's gsplat 1.0.0 kernels compiled from its sources
    (oracle/_ref/gsplat) on the same inputs. Seeded scene: 2 M Gaussians in
    a box in front of a 1920 x 1080 camera, log-normal scales, uniform
    opacities, N(0, 0.2) degree-3 SH coefficients (colors evaluated from them,
    as the engine does). One JSON line per implementation (CUDA events,
    median over --steps after --warmup)."""
    from oracle import build_ref
    from oracle import render as orc
    from tidegs_b200 import render as tr

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    Wd, Hd, tile, n = 1920, 1080, 16, 2_000_000
    g = torch.Generator(device=dev).manual_seed(3)
    means = (torch.rand((n, 3), generator=g, device=dev) * torch.tensor([16.0, 9.0, 20.0], device=dev)
             + torch.tensor([-8.0, -4.5, 4.0], device=dev))
    quats = torch.randn((n, 4), generator=g, device=dev)
    scales = torch.exp(torch.randn((n, 3), generator=g, device=dev) * 0.5 - 3.2)
    opac = torch.rand((1, n), generator=g, device=dev) * 0.9 + 0.05
    # degree-3 SH coefficients (16 per channel), colors evaluated per camera
    coeffs = torch.randn((1, n, 16, 3), generator=g, device=dev) * 0.2
    dirs = (means - torch.tensor([0.0, 0.0, -1.0], device=dev))[None].contiguous()
    view = orc.look_at((0.0, 0.0, -1.0), (0.0, 0.0, 10.0), up=(0.0, -1.0, 0.0))[None].float().to(dev)
    K = orc.intrinsics(Wd, Hd, 70.0)[None].float().to(dev)
    tw, th = (Wd + tile - 1) // tile, (Hd + tile - 1) // tile
    ref = build_ref.load_prebuilt_gsplat()
    means_g, quats_g, scales_g = (t.clone().requires_grad_(True) for t in (means, quats, scales))
    coeffs_g = coeffs.clone().requires_grad_(True)

    def run_ours():
        marks = {}
        radii, m2, dep, con, _ = tr._Projection.apply(means_g, quats_g, scales_g, view, K, Wd, Hd,
                                                      0.3, 0.01, 1e10, 0.0, False)
        marks["projection"] = torch.cuda.Event(enable_timing=True)
        marks["projection"].record()
        sh_out = tr.spherical_harmonics(3, dirs, coeffs_g)
        colors = sh_out.detach()
        marks["sh"] = torch.cuda.Event(enable_timing=True)
        marks["sh"].record()
        _, ids, flat = tr.isect_tiles(m2, radii, dep, tile, tw, th)
        offs = tr.isect_offset_encode(ids, 1, tw, th)
        marks["intersect"] = torch.cuda.Event(enable_timing=True)
        marks["intersect"].record()
        # the raw kernels, called as the reference arm calls its binding
        m2d, cond = m2.detach(), con.detach()
        rc, ra, last = tr.rasterize_to_pixels_fwd(m2d, cond, colors, opac, None, Wd, Hd, tile,
                                                  offs, flat)
        marks["raster_fwd"] = torch.cuda.Event(enable_timing=True)
        marks["raster_fwd"].record()
        _, vm, vc, vcol, _ = tr.rasterize_to_pixels_bwd(m2d, cond, colors, opac, None, Wd, Hd,
                                                        tile, offs, flat, ra, last,
                                                        torch.ones_like(rc), torch.ones_like(ra),
                                                        False)
        marks["raster_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["raster_bwd"].record()
        # autograd.grad: the gradients are returned, not added into the
        # leaves' .grad (an extra pass over them the reference arm does not do)
        torch.autograd.grad([sh_out], [coeffs_g], [vcol])
        marks["sh_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["sh_bwd"].record()
        torch.autograd.grad([m2, dep, con], [means_g, quats_g, scales_g],
                            [vm, torch.zeros_like(dep), vc])
        marks["projection_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["projection_bwd"].record()
        return marks, int(flat.numel())

    def run_ref():
        marks = {}
        radii, m2, dep, con, _ = ref.fully_fused_projection_fwd(means, None, quats, scales, view, K,
                                                                Wd, Hd, 0.3, 0.01, 1e10, 0.0, False)
        marks["projection"] = torch.cuda.Event(enable_timing=True)
        marks["projection"].record()
        colors = ref.compute_sh_fwd(3, dirs, coeffs, None)
        marks["sh"] = torch.cuda.Event(enable_timing=True)
        marks["sh"].record()
        _, ids, flat = ref.isect_tiles(m2, radii, dep, None, None, 1, tile, tw, th, True, True)
        offs = ref.isect_offset_encode(ids, 1, tw, th)
        marks["intersect"] = torch.cuda.Event(enable_timing=True)
        marks["intersect"].record()
        rc, ra, last = ref.rasterize_to_pixels_fwd(m2, con, colors, opac, None, Wd, Hd, tile, offs, flat)
        marks["raster_fwd"] = torch.cuda.Event(enable_timing=True)
        marks["raster_fwd"].record()
        _, vm, vc, vcol, vo = ref.rasterize_to_pixels_bwd(m2, con, colors, opac, None, Wd, Hd, tile,
                                                          offs, flat, ra, last, torch.ones_like(rc),
                                                          torch.ones_like(ra), False)
        marks["raster_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["raster_bwd"].record()
        ref.compute_sh_bwd(16, 3, dirs, coeffs, None, vcol, False)
        marks["sh_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["sh_bwd"].record()
        ref.fully_fused_projection_bwd(means, None, quats, scales, view, K, Wd, Hd, 0.3, radii, con,
                                       None, vm, torch.zeros_like(dep), vc, None, False)
        marks["projection_bwd"] = torch.cuda.Event(enable_timing=True)
        marks["projection_bwd"].record()
        return marks, int(flat.numel())

    arms = [("tidegs_b200", run_ours)]
    if ref is not None:
        arms.append(("reference_gsplat", run_ref))
    for name, fn in arms:
        per = {}
        for k in range(args.warmup + args.steps):
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
            marks, n_isects = fn()
            torch.cuda.synchronize()
            if k < args.warmup:
                continue
            prev = e0
            for stage, ev in marks.items():
                per.setdefault(stage, []).append(prev.elapsed_time(ev))
                prev = ev
        out = {"probe": "render", "impl": name, "gaussians": n, "image": [Wd, Hd],
               "intersections": n_isects}
        out.update({k + "_ms": round(statistics.median(v), 3) for k, v in per.items()})
        out["total_ms"] = round(sum(out[k + "_ms"] for k in per), 3)
        print(json.dumps(out), flush=True)


def accum_probe(args):
    """Not the bench line. A camera batch of the configs[3] shape (16 cameras,
    each seeing a contiguous run of 24-56 resident blocks of 16,384 rows out
    of 2048) accumulated by SparseGradAccumulator, and by the reference's own
    torch operations on the same GPU (engine.py:1801-1826: mask, nonzero,
    zeros; :2434-2471: searchsorted + six scatter_add_ per camera). Checks the
    two results are equal; prints one JSON line (CUDA events, median)."""
    from tidegs_b200 import SparseGradAccumulator

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    M = SLOTS * B
    rng = np.random.default_rng(10_000)
    filters, grads = [], []
    for _ in range(16):
        length = max(1, int(rng.integers(24, 56) * SLOTS / 2048))
        start = int(rng.integers(0, max(1, SLOTS - length)))
        f = torch.arange(start * B, (start + length) * B, dtype=torch.int64, device=dev)
        n = f.numel()
        filters.append(f)
        grads.append({k: torch.empty((n, w), device=dev).normal_(0, 1e-3) for k, w in
                      (("xyz", 3), ("opacity", 1), ("scaling", 3), ("rotation", 4), ("shs", 48))})
    filter_rows = sum(f.numel() for f in filters)

    split = []

    def ours():
        acc = SparseGradAccumulator(filters, M)
        mid = torch.cuda.Event(enable_timing=True)
        mid.record()
        for f, g in zip(filters, grads):
            acc.add(f, g["xyz"], g["opacity"], g["scaling"], g["rotation"], g["shs"])
        split.append(mid)
        return acc.sparse_grad_local_ids, acc.sparse_grad_components

    def reference():
        mask = torch.zeros((M,), dtype=torch.bool, device=dev)
        for f in filters:
            mask.scatter_(0, f, True)
        ids = torch.nonzero(mask, as_tuple=False).flatten()
        n = int(ids.numel())
        comps = {k: torch.zeros((n, w), device=dev) for k, w in WIDTHS.items()}
        for f, g in zip(filters, grads):
            idx = torch.searchsorted(ids, f)
            for k, w in (("xyz", 3), ("opacity", 1), ("scaling", 3), ("rotation", 4)):
                comps[k].scatter_add_(0, idx.reshape(-1, 1).expand(-1, w), g[k])
            comps["features_dc"].scatter_add_(0, idx.reshape(-1, 1).expand(-1, 3), g["shs"][:, :3])
            comps["features_rest"].scatter_add_(0, idx.reshape(-1, 1).expand(-1, 45),
                                                g["shs"][:, 3:48])
        return ids, comps

    out = {}
    adds = []
    for name, fn in (("tidegs_b200", ours), ("reference_torch_ops", reference)):
        times = []
        for k in range(args.warmup + args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            split.clear()
            e0.record()
            res = fn()
            e1.record()
            torch.cuda.synchronize()
            if k >= args.warmup:
                times.append(e0.elapsed_time(e1))
                if split:
                    adds.append(split[0].elapsed_time(e1))
        out[name] = (sorted(times)[len(times) // 2], res)
    (ids_a, ca), (ids_b, cb) = out["tidegs_b200"][1], out["reference_torch_ops"][1]
    equal = bool(torch.equal(ids_a, ids_b)) and all(torch.equal(ca[k], cb[k]) for k in WIDTHS)
    ms = out["tidegs_b200"][0]
    print(json.dumps({"probe": "sparse_grad_accumulation", "cameras": len(filters),
                      "filter_rows": filter_rows, "touched_rows": int(ids_a.numel()),
                      "ms": ms, "reference_torch_ops_ms": out["reference_torch_ops"][0],
                      "equal_to_reference_ops": equal,
                      "accumulate_ms": sorted(adds)[len(adds) // 2],
                      "accumulate_GBps": filter_rows * 712 / (sorted(adds)[len(adds) // 2] / 1e3)
                      / 1e9}), flush=True)
    return 0


# ---------------------------------------------------------------------------
# CPU baseline: the reference's torch CPU path (oracle port), bounded sample
# ---------------------------------------------------------------------------
def cpu_baseline(seconds_budget: float = 12.0):
    from oracle.resident_adam import COMPONENT_SPECS, TorchFallbackResidentAdam
    from oracle import blocks as ob

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    slots = 64                      # 1/32 of a GPU's 2048 slots, same ratios
    Bs = B
    rows = slots * Bs
    opt = TorchFallbackResidentAdam(rows, seed=0)
    rng = np.random.default_rng(0)
    vis = np.sort(rng.choice(slots, int(round(slots * 0.3)), replace=False))
    local = torch.from_numpy((vis[:, None] * Bs + np.arange(Bs)[None, :]).reshape(-1))
    n = local.numel()
    grads = {name: torch.randn((n, w)) * 1e-3 for name, _, w, _ in COMPONENT_SPECS}
    lrs = [LRS[name] for name, _, _, _ in COMPONENT_SPECS]
    slots_of_row = local // Bs
    turnover = slots // 4
    packed_in = torch.randn((turnover * Bs, 59))
    done_rows = 0
    t0 = time.perf_counter()
    steps = 0
    while True:
        opt.step(local, local, slots_of_row, grads, lrs, slots, step=steps + 1, batch_size=16)
        # materialization + write-back of the same sample (torch CPU copies,
        # as the reference's fallback paths do them)
        ev = np.sort(rng.choice(slots, turnover, replace=False))
        for i, s in enumerate(ev):
            src = packed_in[i * Bs:(i + 1) * Bs]
            for name, (a, w) in (("xyz", (0, 3)), ("scaling", (3, 3)), ("rotation", (6, 4)),
                                 ("opacity", (10, 1)), ("features_dc", (11, 3)),
                                 ("features_rest", (14, 45))):
                opt.params[name][s * Bs:(s + 1) * Bs].copy_(src[:, a:a + w])
        dirty = ev[: turnover // 2]
        torch.cat([torch.cat([opt.params[nm][s * Bs:(s + 1) * Bs] for nm in
                              ("xyz", "scaling", "rotation", "opacity", "features_dc",
                               "features_rest")], dim=1) for s in dirty])
        done_rows += n
        steps += 1
        if time.perf_counter() - t0 > seconds_budget:
            break
    elapsed = time.perf_counter() - t0
    return {
        "value": done_rows / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
        # one full-size step (SLOTS slots) at the sample's rate
        "ms_per_step": 1e3 * (n * SLOTS / slots) / (done_rows / elapsed),
        "sample": (f"{slots} slots x {Bs} rows (1/32 of a GPU's resident set), 30% blocks "
                   f"visible ({n} rows), 25% turnover, {steps} steps in {elapsed:.1f} s: "
                   "reference torch CPU step (gpu_resident_optimizer.py:339-364 ported), "
                   "slot fill and write-back pack by torch copies"),
    }


# ---------------------------------------------------------------------------
def run_reference_arm(args, world, rank):
    if rank != 0:
        return 0
    budget = max(1.0, 20.0 / max(1, args.steps + args.warmup))
    base = cpu_baseline(seconds_budget=budget * max(1, args.steps))
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE configs[3] shapes and distributions)",
        "config": dict(WORKLOAD_CONFIG, slots_per_gpu=SLOTS, block_size=B,
                       turnover_blocks=TURNOVER,
                       run="the reference's CPU step on a bounded sample of this workload "
                           "(cpu_baseline.sample), all host threads, rank 0 only"),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tidegs_b200", choices=["tidegs_b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--e2e-warmup", type=int, default=6)
    ap.add_argument("--e2e-profile", action="store_true",
                    help="print a per-phase wall-time breakdown of the e2e step to stderr")
    ap.add_argument("--pool-blocks", type=int, default=1024,
                    help="distinct seeded host blocks (scene block b holds block b mod this)")
    ap.add_argument("--host-tier", default="cache", choices=["cache", "pool"],
                    help="e2e host side: PinnedBlockCache over every scene block of the rank "
                         "(write-back lands in it), or the fixed modulo PinnedBlockPool")
    ap.add_argument("--slots", type=int, default=SLOTS,
                    help="resident slots per GPU (default: the configs[3] value; smaller "
                         "values make small profiling cases of the same step)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--phase-times", action="store_true",
                    help="print a per-phase CUDA-event breakdown of the device step to stderr "
                         "(extra events; not used for the reported value)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pull-probe", default=None, metavar="MODES",
                    help="diagnostic instead of the bench: comma list of remote,local,plain "
                         "(needs two GPUs for remote)")
    ap.add_argument("--cull-probe", action="store_true",
                    help="diagnostic: frustum culling of a 61,036-block scene, 16 cameras")
    ap.add_argument("--render-probe", action="store_true",
                    help="diagnostic: render path, ours vs the reference gsplat kernels")
    ap.add_argument("--accum-probe", action="store_true",
                    help="diagnostic instead of the bench: touched-only gradient accumulation "
                         "of a camera batch against the reference's torch operations")
    ap.add_argument("--exchange", default="pull", choices=["pull", "push", "nccl"],
                    help="N>1 gradient exchange: the owner's update kernel sums the senders' "
                         "gradients over NVLink (pull, default); a push kernel into receive "
                         "buffers + owner sum (push); or pack + NCCL all-to-all + owner sum")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)
    set_slots(args.slots)
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference_arm(args, world, rank)
    if args.pull_probe:
        return pull_probe(args, args.pull_probe.split(","))
    if args.accum_probe:
        return accum_probe(args)
    if args.cull_probe:
        return cull_probe(args)
    if args.render_probe:
        return render_probe(args)

    from tidegs_b200 import _lib

    device = torch.device("cuda", torch.cuda.current_device())
    global POOL_MULT
    POOL_MULT, args.host_tier = plan_host_pool(world, args.host_tier, args.pool_blocks,
                                               host_memory_limit())
    n_trace = max(args.warmup + args.steps + 3, args.e2e_warmup + args.e2e_steps + 1)
    trace = ScheduleTrace(world, rank, n_trace)
    scheds = [Schedule(o, world) for o in range(world)]
    sched = scheds[rank]
    dev = DeviceStep(device, sched, trace, scheds=scheds, world=world, exchange=args.exchange)
    for k in range(args.warmup):
        dev.step(k)
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(device)
    launches0 = _lib.launch_counter["kernels"]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    rows = 0
    for k in range(args.warmup, args.warmup + args.steps):
        rows += dev.step(k, timed=True)
    end.record()
    torch.cuda.synchronize()
    if args.phase_times:
        # separate, untimed pass: per-phase CUDA events around each stage
        dev.phase_ms, dev.host_ms = {}, {}
        for k in range(args.warmup + args.steps, args.warmup + args.steps + 3):
            dev.step(k)
            dev.collect_phases()
        print(f"rank {rank} device phase ms/step: " + json.dumps(
            {n: round(sum(v) / len(v), 3) for n, v in dev.phase_ms.items()})
            + " host ms/step: " + json.dumps(
            {n: round(sum(v) / len(v), 3) for n, v in dev.host_ms.items()}),
            file=sys.stderr, flush=True)
        dev.phase_ms = dev.host_ms = None
    barrier(world)
    clock_info = clocks.stop()
    launches = _lib.launch_counter["kernels"] - launches0
    ms = start.elapsed_time(end)
    ms_max = allreduce_max(ms, world)
    total_rows = rows * world
    value = total_rows / (ms_max / 1e3)
    adam_ms, adam_rows = dev.adam_stats()
    adam_avg_ms = sum(adam_ms) / len(adam_ms)
    adam_max_ms = allreduce_max(adam_avg_ms, world)
    adam_bytes = ADAM_BYTES_PER_ROW * (sum(adam_rows) / len(adam_rows))
    achieved = adam_bytes / (adam_avg_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    exchange_rows = getattr(dev, "exchange_rows", 0)
    dev.close()
    del dev
    torch.cuda.empty_cache()

    # e2e leg through the Python API (host pool -> HBM -> host)
    e2e = None
    try:
        if args.no_e2e:
            raise _Skipped("--no-e2e")
        api = ApiStep(device, [Schedule(o, world) for o in range(world)], trace, rank, world,
                      args.pool_blocks, exchange=args.exchange, host_tier=args.host_tier)
        for k in range(args.e2e_warmup):
            api.step(k)
        torch.cuda.synchronize()
        barrier(world)
        api.h2d_bytes = api.d2h_bytes = 0
        api.profile = {} if args.e2e_profile else None
        e_rows = 0
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for k in range(args.e2e_warmup, args.e2e_warmup + args.e2e_steps):
            e_rows += api.step(k)
        t1.record()
        torch.cuda.synchronize()
        e_ms = allreduce_max(t0.elapsed_time(t1), world)
        e2e = {"value": e_rows * world / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int(api.h2d_bytes / args.e2e_steps),
               "d2h_bytes_per_step": int(api.d2h_bytes / args.e2e_steps),
               "ms_per_step": e_ms / args.e2e_steps, "steps": args.e2e_steps,
               "host_pool_blocks": args.pool_blocks,
               "host_tier": (f"PinnedBlockCache of the rank's {POOL_MULT * SLOTS} scene blocks "
                             f"(+{TURNOVER} write-back entries); write-back DMA into it"
                             if args.host_tier == "cache" else
                             f"PinnedBlockPool of {args.pool_blocks} blocks (block id mod pool)")}
        if api.profile is not None and rank == 0:
            print("e2e phase wall ms/step: " + json.dumps(
                {k: round(v * 1e3 / args.e2e_steps, 2) for k, v in api.profile.items()})
                + " writeback staging bytes: "
                + str(api.ws.writeback_stats["pinned_staging_bytes"]),
                file=sys.stderr, flush=True)
        api.close()
        del api
    except _Skipped as why:
        e2e = {"value": None, "unit": UNIT, "skipped": str(why)}
    except Exception as exc:  # report, never hide
        e2e = {"value": None, "unit": UNIT, "error": f"{type(exc).__name__}: {exc}"}

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, BASELINE configs[3] shapes and distributions)",
            "config": {**WORKLOAD_CONFIG,
                       "slots_per_gpu": SLOTS, "block_size": B, "turnover_blocks": TURNOVER,
                       "scene_blocks_per_gpu": POOL_MULT * SLOTS,
                       "rows_updated_per_step": rows / args.steps,
                       "parallelism": f"block ownership, rank = block_id mod {world}",
                       "exchange_rows_per_step": exchange_rows / (args.warmup + args.steps),
                       "exchange": (None if world == 1 else
                                    "owner update kernel sums senders' gradients over NVLink "
                                    "(tgs_resident_adam_apply_sum)" if args.exchange == "pull"
                                    else "direct NVLink push (tgs_grad_push) + ordered owner sum"
                                    if args.exchange == "push" else
                                    "pack + NCCL all-to-all + ordered owner sum"),
                       "l2": "every input larger than L2 (126 MB)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": ADAM_TRAFFIC_BYTES_PER_ROW * (sum(adam_rows) / len(adam_rows)),
                         "traffic_note": "bytes per launch: ncu DRAM bytes per row of the "
                                         "256-slot capture x rows per launch",
                         "kernel": "resident_adam_kernel",
                         "algorithmic_bytes_per_row": ADAM_BYTES_PER_ROW,
                         "avg_launch_ms": adam_avg_ms, "peak_source": peak_kind,
                         "avg_launch_ms_max_over_ranks": adam_max_ms},
            "clocks": clock_info,
            "gpu_launches": launches,
            "e2e": e2e,
            "cpu_baseline": base,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
