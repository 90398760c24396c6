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
  4. materialization of 512 incoming blocks (packed rows -> component arrays
     + global ids) straight into the spare slots of the slot arena, whose
     evicted slots become the next spare ones (no slot-remap copy). The
     unpack is enqueued before the pack: it does not depend on the
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


def plan_host_tier(world: int, host_tier: str, pool_blocks: int, host_blocks: int,
                   limit: int) -> str:
    """The e2e leg's host tier: a page-locked cache of every block the rank
    holds during the e2e steps (plus one write-back batch and the seeded
    source blocks) while all ranks' caches fit in 60 % of the box's memory,
    else the small fixed page-locked pool (block id mod pool_blocks)."""
    budget = 0.6 * limit / world
    if host_tier == "cache" and (host_blocks + TURNOVER + pool_blocks) * BLOCK_BYTES > budget:
        return "pool"
    return host_tier


WORKLOAD_CONFIG = {
    "workload": "configs[4] block schedule: 61,036-block scene (1.0 B Gaussians), owner = "
                "block_id mod N, 2048 resident slots x 16384 Gaussians per GPU, one 16-camera "
                "batch per step split across the ranks on a smooth trajectory (neighbouring "
                "cameras share 70% of their blocks; the batch sees ~30% of every owner's "
                "slots), 25% slot turnover per step, dirty blocks written back; at N=1 this "
                "is configs[3]'s full resident-set step"}

WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}
NAMES = tuple(WIDTHS)
ADAM_BYTES_PER_ROW = 59 * 4 * 7          # grad r + param r/w + m r/w + v r/w
# DRAM bytes per updated row of resident_adam_stream_kernel measured by ncu:
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the 256-slot
# step (every input larger than L2) = 1194.0 MB + 852.2 MB over its
# 1,212,416 rows
ADAM_TRAFFIC_BYTES_PER_ROW = 1687.7
# NVLink bandwidth per direction of one B200 measured on this box type (peer
# copy), the denominator of the parameter gather's fraction
NVLINK_GBPS = 770.0
# From this many ranks `--overlap auto` runs the block materialization beside
# the pull update, on the SMs the update leaves free (OVERLAP_ADAM_CTAS of
# 148 for the update): where NVLink bounds the update (remote contributions
# per owner grow with the camera split), HBM has room for it. Measured on
# B200 (G updates/s, update CTAs): 8 GPUs 10.67 without the overlap, 10.86
# (148), 11.50 (128), 11.97 (120), 12.48 (112), 12.24 (96), 11.33 (80);
# 4 GPUs 7.47 without, 7.68 (128), 7.86 (112), 7.23 (96); 2 GPUs 4.16
# without, 3.99 (112): there the step is HBM-bound.
OVERLAP_MIN_WORLD = 4
OVERLAP_ADAM_CTAS = 112
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


def _gather_all(obj, world: int) -> list:
    """Every rank's `obj`, in rank order (a plain list at world 1)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


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
        # nvidia-smi takes a while to start (longer with one instance per
        # rank); keep it until it has written a sample, at most 5 s
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            try:
                if Path(self.path).read_text().count("\n") >= 1:
                    break
            except OSError:
                pass
            time.sleep(0.05)
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
# Workload generation: BASELINE configs[4]'s block schedule (seeded)
# ---------------------------------------------------------------------------
SCENE_BLOCKS = 61036   # 1,000,013,824 Gaussians in 16,384-row blocks
CAMERAS = 16           # camera batch per step, split across the ranks
VISIBLE_FRAC = 0.30    # the batch sees ~30 % of every owner's resident slots
OVERLAP = 0.70         # neighbouring cameras share 70 % of their blocks


class Trajectory:
    """The camera schedule all ranks share. Blocks are numbered along the
    scene's space-filling order, so a camera sees a contiguous run of block
    ids. Each step one batch of CAMERAS cameras sits on a smooth path: camera
    i's run starts (1 - OVERLAP) of a run after camera i-1's, so neighbours
    share OVERLAP of their blocks, and the batch's union covers VISIBLE_FRAC
    of the resident window. The resident window (SLOTS * world consecutive
    block ids, SLOTS of them owned by each rank under owner = id mod world)
    follows the batch by TURNOVER * world ids a step, bouncing at the ends of
    the scene, so every owner turns over exactly TURNOVER slots a step.
    Rank r renders cameras [CAMERAS*r/world, CAMERAS*(r+1)/world)."""

    def __init__(self, world: int, seed: int = 4):
        if CAMERAS % world:
            raise ValueError(f"{CAMERAS} cameras do not split across {world} ranks")
        self.world = world
        self.span = SLOTS * world
        self.shift = TURNOVER * world
        if self.span > SCENE_BLOCKS:
            raise ValueError("resident window larger than the scene")
        self.union = max(CAMERAS, int(round(VISIBLE_FRAC * self.span)))
        # union = cam + (CAMERAS - 1) * (1 - OVERLAP) * cam
        self.cam = max(1, int(round(self.union / (1 + (CAMERAS - 1) * (1 - OVERLAP)))))
        self.stride = max(1, int(round((1 - OVERLAP) * self.cam)))
        self.extent = self.cam + (CAMERAS - 1) * self.stride
        self.n_pos = (SCENE_BLOCKS - self.span) // self.shift  # window positions 0..n_pos
        self.seed = seed

    def start(self, k: int) -> int:
        """First block id of the resident window at step k (back and forth)."""
        if self.n_pos == 0:
            return 0
        j = k % (2 * self.n_pos)
        return self.shift * (j if j <= self.n_pos else 2 * self.n_pos - j)

    def cameras(self, k: int):
        """[lo, hi) block-id runs of the batch's cameras at step k."""
        slack = self.span - self.extent
        # the batch drifts smoothly inside the window around its centre
        off = slack // 2 + int(round(0.25 * slack * math.sin(0.37 * k + self.seed)))
        lo0 = self.start(k) + max(0, min(slack, off))
        return [(lo0 + i * self.stride, lo0 + i * self.stride + self.cam) for i in range(CAMERAS)]

    def rendered(self, k: int, rank: int) -> np.ndarray:
        """Block ids rank `rank`'s cameras see at step k (ascending)."""
        per = CAMERAS // self.world
        runs = self.cameras(k)[rank * per:(rank + 1) * per]
        return np.arange(runs[0][0], runs[-1][1], dtype=np.int64)

    def visible(self, k: int) -> np.ndarray:
        runs = self.cameras(k)
        return np.arange(runs[0][0], runs[-1][1], dtype=np.int64)

    def max_owned_visible(self) -> int:
        """Upper bound of one owner's visible blocks in any step."""
        return -(-self.extent // self.world) + 1


class Schedule:
    """One owner's resident slots along the trajectory: slot position i
    holds block slot_block[i]; incoming blocks (ascending) take the freed
    positions (ascending), the persistent-slot plan's rule."""

    def __init__(self, rank: int, world: int, traj: "Trajectory" = None):
        self.traj = traj if traj is not None else Trajectory(world)
        self.world, self.rank = world, rank
        a = self.traj.start(0)
        self.slot_block = self.owned(a, a + self.traj.span)
        assert self.slot_block.size == SLOTS
        self.num_blocks = SCENE_BLOCKS

    def owned(self, lo: int, hi: int) -> np.ndarray:
        first = lo + (self.rank - lo) % self.world
        return np.arange(first, hi, self.world, dtype=np.int64)

    def slot_table(self) -> np.ndarray:
        """Dense block id -> slot position table (-1: not resident)."""
        table = np.full(SCENE_BLOCKS, -1, np.int64)
        table[self.slot_block] = np.arange(self.slot_block.size, dtype=np.int64)
        return table

    def visible_blocks(self, k: int) -> np.ndarray:
        """This owner's blocks the batch of step k sees (ascending id)."""
        v = self.traj.visible(k)
        return v[v % self.world == self.rank]

    def visible_positions(self, k: int) -> np.ndarray:
        """Slot positions of this owner's visible blocks at step k, ascending
        (the owner's row ids are all rows of these positions)."""
        pos = self.slot_table()[self.visible_blocks(k)]
        if pos.size and pos.min() < 0:
            raise RuntimeError("a visible block is not resident")
        return np.sort(pos)

    def turnover(self, k: int):
        """(evicted positions ascending, incoming block ids ascending, None)
        between steps k and k+1; the blocks' dirty state decides the
        write-back."""
        a0, a1 = self.traj.start(k), self.traj.start(k + 1)
        span = self.traj.span
        if a1 >= a0:
            leaving, entering = self.owned(a0, a1), self.owned(a0 + span, a1 + span)
        else:
            leaving, entering = self.owned(a1 + span, a0 + span), self.owned(a1, a0)
        evict_pos = np.sort(self.slot_table()[leaving])
        return evict_pos, entering, None

    def touched_blocks(self, n_steps: int) -> np.ndarray:
        """Every block this owner holds during steps [0, n_steps]."""
        starts = [self.traj.start(k) for k in range(n_steps + 1)]
        return self.owned(min(starts), max(starts) + self.traj.span)


class RandomTurnover:
    """configs[2]'s materialization schedule over one owner's slot map: each
    iteration TURNOVER random slots take random non-resident blocks of a
    host pool (random block-id -> slot remap), Bernoulli(0.5) dirty flags on
    the evicted blocks."""

    def __init__(self, slot_block: np.ndarray, pool_ids: np.ndarray, seed: int = 3):
        self.slot_block = slot_block
        self.pool_ids = np.sort(np.asarray(pool_ids, np.int64))
        self.seed = seed

    def turnover(self, k: int):
        rng = np.random.default_rng(self.seed * 100_003 + k)
        evict_pos = np.sort(rng.choice(self.slot_block.size, TURNOVER, replace=False))
        resident = np.isin(self.pool_ids, self.slot_block, assume_unique=True)
        incoming = np.sort(rng.choice(self.pool_ids[~resident], TURNOVER, replace=False))
        return evict_pos, incoming, rng.random(TURNOVER) < 0.5


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
def rendered_blocks(traj: "Trajectory", step: int, world: int):
    """Block ids whose gradients each rank renders at `step`."""
    return [traj.rendered(step, r) for r in range(world)]


def exchange_capacity(sched: "Schedule", world: int, n_steps: int):
    """(blocks a rank renders, tiles an owner receives): the largest over
    the steps of the trace."""
    send_max = recv_max = 0
    for k in range(n_steps):
        ren = rendered_blocks(sched.traj, k, world)
        send_max = max(send_max, ren[sched.rank].size)
        recv_max = max(recv_max, sum(int(np.count_nonzero(r % world == sched.rank))
                                     for r in ren))
    return send_max, recv_max


class ScheduleTrace:
    """The synthetic schedule simulated ahead of the timed region (workload
    generation, not the measured path): for step k, the blocks each rank
    renders (vis[k], world > 1) and this rank's slot turnover (turn[k] =
    evicted slot positions, incoming block ids, dirty pattern or None)."""

    def __init__(self, world: int, rank: int, n_steps: int):
        traj = Trajectory(world)
        sched = Schedule(rank, world, traj)
        self.n_steps = n_steps
        self.vis, self.turn = [], []
        for k in range(n_steps):
            self.vis.append(rendered_blocks(traj, k, world) if world > 1 else None)
            ev, inc, dirty = sched.turnover(k)
            self.turn.append((ev, inc, dirty))
            sched.slot_block[ev] = inc


class DeviceStep:
    """The step through the library entry points, every input in HBM. The
    resident blocks live in a slot arena of SLOTS + TURNOVER block slots:
    the TURNOVER spare slots receive the next step's incoming blocks straight
    from the unpack (tgs_unpack_rows' block scatter), and the evicted blocks'
    slots become the spare ones, so no slot-remap copy is needed. A block's
    optimizer state lives with its arena slot (state slot = arena slot): a
    block keeps its slot while resident, and an incoming block's slot gets a
    new admission stamp (its moments read as zero)."""

    def __init__(self, device, sched: Schedule, trace: ScheduleTrace, world: int = 1,
                 exchange: str = "pull", overlap: bool = False, adam_ctas: int = 0):
        from tidegs_b200 import _lib, _ops

        self._lib, self._ops = _lib, _ops
        self.device = device
        self.sched = sched
        self.trace = trace
        self.world = world
        gen = torch.Generator(device=device).manual_seed(1234 + sched.rank)
        self.n_arena = SLOTS + TURNOVER
        rows = self.n_arena * B
        # schedule position i -> arena slot; arena slot -> block (-1 spare)
        self.arena_of_pos = np.arange(SLOTS, dtype=np.int64)
        self.arena_block = np.full(self.n_arena, -1, np.int64)
        self.arena_block[:SLOTS] = sched.slot_block
        self.spare = np.arange(SLOTS, self.n_arena, dtype=np.int64)
        self.arena = {n: torch.empty((rows, w), device=device) for n, w in WIDTHS.items()}
        fill_params(self.arena, gen)
        self.gids = torch.empty(rows, dtype=torch.int64, device=device)
        _ops.fill_global_ids(self.gids, 0, _ops.i64_to_device(self.arena_block, device), rows, B)
        # incoming blocks already landed in HBM (packed CACHE rows), 2 rotating sets
        self.incoming_pool = torch.empty((2 * TURNOVER * B, 59), device=device)
        self.incoming_pool.normal_(0.0, 1.0, generator=gen)
        self.wb_staging = torch.empty((TURNOVER * B, 59), device=device)
        self.bounds = torch.empty((self.n_arena, 6), device=device)
        # resident Adam state, one optimizer slot per arena slot
        self.state = torch.zeros((rows, 128), device=device)
        self.slot_step = torch.zeros(self.n_arena, dtype=torch.int32, device=device)
        self.stamp_host = np.ones(self.n_arena, np.uint32)
        self.slot_stamp = torch.ones(self.n_arena, dtype=torch.int32, device=device)
        self.slot_bias = torch.ones((self.n_arena, 2), device=device)
        table = [(0.0, 0.0)] + [(float(np.float32(1 - 0.9 ** t)),
                                 float(np.float32(math.sqrt(1 - 0.999 ** t))))
                                for t in range(1, 20000)]
        self.table = torch.tensor(table, dtype=torch.float32, device=device)
        self.err = torch.zeros(4, dtype=torch.int32, device=device)
        self.pos_count = torch.zeros(self.n_arena, dtype=torch.int32, device=device)
        self.chunk_table = torch.empty(2 * sched.traj.max_owned_visible() * B // 32,
                                       dtype=torch.int64, device=device)
        # working-set positions = arena slots; a spare slot is an empty slice
        self.pos_start_host = np.arange(self.n_arena, dtype=np.int64) * B
        self.pos_start = _ops.i64_to_device(self.pos_start_host, device)
        self.pos_end = torch.empty(self.n_arena, dtype=torch.int64, device=device)
        self._upload_pos_end()
        self.pos_slot = torch.arange(self.n_arena, dtype=torch.int32, device=device)
        self.bitmap = torch.zeros(_ops.bitmap_words(SCENE_BLOCKS), dtype=torch.int32,
                                  device=device)
        # the owner's row ids of a step (all rows of its visible positions)
        # are expanded on the device from the positions; gradients of the
        # largest step
        max_rows = sched.traj.max_owned_visible() * B
        self.ids_buf = torch.empty(max_rows, dtype=torch.int64, device=device)
        self.grads = {n: torch.empty((max_rows, w), device=device).normal_(0, 1e-3, generator=gen)
                      for n, w in WIDTHS.items()}
        self.exchange_mode = exchange if world > 1 else None
        self.peer = None
        self.pull = None
        self.plan = None
        if world > 1:
            # gradients this rank renders for blocks of every owner, and the
            # exchange buffers (sizes: the largest of the periodic camera sets)
            send_max, recv_max = exchange_capacity(sched, world, trace.n_steps)
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
            # updated parameters reach the ranks that render the blocks next
            from tidegs_b200.sharded import PeerParamGather

            self.param_gather = PeerParamGather(self.arena, B, device)
        self.adam_ms = []
        self.updated_rows = []
        # pipelined materialization: step k's write-back of step k-1's dirty
        # evicted blocks and its unpack of the incoming blocks run on a side
        # stream while the update runs on the main one (step_overlapped)
        self.overlap = bool(overlap)
        self.adam_ctas = int(adam_ctas)
        if self.overlap:
            self.side = torch.cuda.Stream(device)
            self.ev_main = torch.cuda.Event()   # update + bounds of the last step done
            self.ev_side = torch.cuda.Event()   # unpack of the last step landed
            self.ev_main.record()
            self.ev_side.record()
            self._pending_wb = None             # (selection, evicted blocks, slots) of step k-1
        torch.cuda.synchronize()

    def _upload_pos_end(self) -> None:
        """Working-set slices: a resident arena slot covers its B rows, a
        spare one is empty (no row id can fall in it)."""
        end = self.pos_start_host + np.where(self.arena_block >= 0, B, 0)
        self._ops.upload_into(self.pos_end, end)

    def visible_arena(self, k: int) -> np.ndarray:
        """Arena slots of this owner's visible blocks at step k, ascending
        (the owner's row ids are all rows of these slots, in this order)."""
        return np.sort(self.arena_of_pos[self.sched.visible_positions(k)])

    def exchange_grads(self, k: int):
        """Owner-sharded gradient exchange of step k (world > 1): returns the
        owner's visible arena slots and local row ids; the reduced gradients
        land in self.grads (or are summed by the pull kernel)."""
        W, me = self.world, self.sched.rank
        vis = self.trace.vis[k]
        if self._ahead is not None and self._ahead[0] == k:
            _, plan, slot_of, self.pull_tables = self._ahead  # built during step k-1
        else:
            plan, slot_of, self.pull_tables = self._make_plan(k, self.arena_block)
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
        slots = slot_of[plan.out_blocks]
        # the plan's output blocks are the owner's visible blocks in slot order
        if not np.array_equal(slots, self.visible_arena(k)):
            raise RuntimeError("exchange plan and owner visibility disagree")
        return slots, self.row_ids(slots)

    def row_ids(self, slots: np.ndarray) -> torch.Tensor:
        """All rows of arena slots `slots` (ascending), expanded on the
        device from the slots."""
        n = int(slots.size) * B
        if n > self.ids_buf.numel():
            raise RuntimeError(f"{slots.size} visible blocks exceed the row-id buffer")
        ids = self.ids_buf[:n]
        self._ops.fill_global_ids(ids, 0, self._ops.i64_to_device(slots, self.device), n, B)
        return ids

    def _make_plan(self, k: int, arena_block: np.ndarray):
        """Exchange plan of step k for the arena map `arena_block` (output
        blocks ordered by arena slot) and, for the pull exchange, its device
        tables."""
        from tidegs_b200.sharded import make_plan

        table = np.full(SCENE_BLOCKS, -1, np.int64)
        held = np.nonzero(arena_block >= 0)[0]
        table[arena_block[held]] = held
        plan = make_plan(self.trace.vis[k], self.world, self.sched.rank, B, out_order=table)
        tables = self.pull.tables(plan) if self.pull is not None else None
        return plan, table, tables

    def _after_turnover(self, k: int):
        """(arena map, position map, spare slots) after step k's turnover:
        position ev[i] takes incoming[i] into spare slot i (both ascending)."""
        ev, inc, _ = self.trace.turn[k]
        arena_block = self.arena_block.copy()
        arena_of_pos = self.arena_of_pos.copy()
        freed = arena_of_pos[ev]
        arena_block[freed] = -1
        arena_block[self.spare] = inc
        arena_of_pos[ev] = self.spare
        return arena_block, arena_of_pos, np.sort(freed)

    def _turn_over(self, k: int, evict_pos: np.ndarray, incoming: np.ndarray) -> None:
        """The spare slots hold step k's incoming blocks and the evicted
        blocks' slots become the spare ones (no copy); the incoming slots get
        new admission stamps (their moments read as zero) and step counters
        of zero, and the working-set slices follow."""
        _ops = self._ops
        new_slots = self.spare
        self.arena_block, self.arena_of_pos, self.spare = self._after_turnover(k)
        self.sched.slot_block[evict_pos] = incoming
        self.stamp_host[new_slots] += 1
        _ops.upload_into(self.slot_stamp, self.stamp_host.view(np.int32))
        self.slot_step.index_fill_(0, _ops.i64_to_device(new_slots, self.device), 0)
        self._upload_pos_end()

    def plan_ahead(self, k: int):
        """Builds step k+1's plan on the host while the GPU runs step k (the
        arena map after step k's turnover is known from the schedule)."""
        if self.world == 1 or k + 1 >= len(self.trace.turn):
            return
        self._ahead = (k + 1,) + self._make_plan(k + 1, self._after_turnover(k)[0])

    _ahead = None
    pull_tables = None

    def adam(self, ids: torch.Tensor, timed: bool):
        _lib = self._lib
        n = ids.numel()
        stream = _lib.stream_handle(self.device)
        c = _lib.ResidentCountArgs(
            pos_start=self.pos_start.data_ptr(), pos_end=self.pos_end.data_ptr(),
            pos_slot=self.pos_slot.data_ptr(), n_positions=self.n_arena, block_size=B,
            param_rows=self.n_arena * B, local_ids=ids.data_ptr(), n_rows=n,
            slot_step=self.slot_step.data_ptr(), slot_stamp=self.slot_stamp.data_ptr(),
            slot_bias=self.slot_bias.data_ptr(), step_table=self.table.data_ptr(),
            step_table_len=self.table.shape[0], n_slots=self.n_arena,
            pos_count=self.pos_count.data_ptr(), err=self.err.data_ptr(),
            chunk_table=self.chunk_table.data_ptr())
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
        a.n_positions, a.block_size = self.n_arena, B
        a.local_ids, a.n_rows = ids.data_ptr(), n
        a.state, a.slot_stamp = self.state.data_ptr(), self.slot_stamp.data_ptr()
        a.slot_bias, a.err = self.slot_bias.data_ptr(), self.err.data_ptr()
        a.chunk_table = self.chunk_table.data_ptr()
        if self.pull is not None:
            self.pull.barrier()  # every rank's gradients of this step are written
            self._phase("acquire")
        if timed:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        if self.pull is not None:
            self.pull.launch(a, self.plan, stream, tables=tables, max_ctas=self.adam_ctas)
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
        if self._side_events is not None:
            s0, s1 = self._side_events
            self.phase_ms.setdefault("side_pack_unpack", []).append(s0.elapsed_time(s1))
            self._side_events = None

    def step(self, k: int, timed: bool = False) -> int:
        if self.overlap:
            return self.step_overlapped(k, timed)
        _ops = self._ops
        self._events = []
        self._phase("start")
        if self.world > 1:
            # 0. gradients of blocks rendered on other ranks reach their owners
            slots, ids = self.exchange_grads(k)
            self._phase("exchange")
        else:
            slots = self.visible_arena(k)
            ids = self.row_ids(slots)
        # 1. optimizer over the visible rows
        self.adam(ids, timed)
        self.plan_ahead(k)
        # 2. updated blocks are dirty; refresh their bounds
        _ops.dirty_mark(self.bitmap, self.arena_block[slots].tolist(), True)
        _ops.block_bounds(self.arena["xyz"], (slots * B).tolist(), [B] * slots.size,
                          self.bounds[: slots.size])
        self._phase("dirty_bounds")
        # 3. evict TURNOVER blocks: write back the dirty ones
        evict_pos, incoming, dirty = self.trace.turn[k]
        evict_slots = self.arena_of_pos[evict_pos]
        evicted_blocks = self.arena_block[evict_slots]
        if dirty is not None:
            # a schedule with a prescribed dirty pattern
            _ops.dirty_mark(self.bitmap, evicted_blocks[dirty].tolist(), True)
            _ops.dirty_mark(self.bitmap, evicted_blocks[~dirty].tolist(), False)
        order = np.argsort(evicted_blocks, kind="stable")
        selection = _ops.dirty_select_async(self.bitmap, evicted_blocks[order].tolist())
        self._phase("dirty_select")
        # 4. materialize the incoming blocks straight into the spare slots
        # (with their global ids); this does not depend on the write-back, so
        # the device runs it while the host waits for the dirty list
        src = self.incoming_pool[(k % 2) * TURNOVER * B:(k % 2 + 1) * TURNOVER * B]
        ids_dev = _ops.i64_to_device(incoming, self.device)
        _ops.unpack_rows(src, self._lib.LAYOUT_CACHE, self.arena, 0, global_ids=self.gids,
                         block_ids=ids_dev, block_size=B, block_dst=self.spare * B)
        self._phase("unpack")
        wb_ids = selection.wait()
        sorted_blocks = evicted_blocks[order]
        wb_slots = evict_slots[order][np.searchsorted(sorted_blocks,
                                                      np.asarray(wb_ids, np.int64))]
        _ops.pack_rows(self.arena, (wb_slots * B).tolist(), [B] * wb_slots.size,
                       self.wb_staging[: wb_slots.size * B], self._lib.LAYOUT_CACHE)
        self._phase("pack")
        _ops.dirty_mark(self.bitmap, wb_ids, False)
        self._phase("writeback")
        # 5. the spare slots hold the incoming blocks; the evicted blocks'
        # slots become the spare ones (no copy). Incoming slots: new stamps.
        self._turn_over(k, evict_pos, incoming)
        self._phase("tables")
        return int(ids.numel())

    def step_overlapped(self, k: int, timed: bool = False) -> int:
        """Step k with the block materialization pipelined beside the update.
        Side stream: write back step k-1's dirty evicted blocks (they left
        the working set at the end of step k-1, after their last update),
        then unpack step k's incoming blocks into the spare slots, which are
        the slots those blocks left. Main stream: the update of step k,
        dirty marks and bounds. Neither touches the other's slots. Step k+1's
        update waits for step k's unpack; step k+1's write-back waits for
        step k's update. The host queues the update first and the side
        stream's work after it, so the main stream never idles while the host
        prepares the write-back. Per step the same kernels run as in step();
        a step writes back the blocks the step before it evicted."""
        _ops = self._ops
        main = torch.cuda.current_stream(self.device)
        self._events = []
        self._phase("start")
        main.wait_event(self.ev_side)     # step k-1's incoming blocks have landed
        self.side.wait_event(self.ev_main)  # step k-1's update and bounds are done
        evict_pos, incoming, dirty = self.trace.turn[k]
        evict_slots = self.arena_of_pos[evict_pos]
        evicted_blocks = self.arena_block[evict_slots]
        if self.world > 1:
            slots, ids = self.exchange_grads(k)
            self._phase("exchange")
        else:
            slots = self.visible_arena(k)
            ids = self.row_ids(slots)
        self.adam(ids, timed)
        # the side stream's work, queued while the GPU runs the update
        pending = self._pending_wb
        wb_ids = pending[0].wait() if pending is not None else []
        with torch.cuda.stream(self.side):
            if self.phase_ms is not None:
                s0 = torch.cuda.Event(enable_timing=True)
                s0.record()
            if pending is not None and len(wb_ids):
                _, sorted_blocks, sorted_slots = pending
                wb_slots = sorted_slots[np.searchsorted(sorted_blocks,
                                                        np.asarray(wb_ids, np.int64))]
                _ops.pack_rows(self.arena, (wb_slots * B).tolist(), [B] * wb_slots.size,
                               self.wb_staging[: wb_slots.size * B], self._lib.LAYOUT_CACHE)
            src = self.incoming_pool[(k % 2) * TURNOVER * B:(k % 2 + 1) * TURNOVER * B]
            ids_dev = _ops.i64_to_device(incoming, self.device)
            _ops.unpack_rows(src, self._lib.LAYOUT_CACHE, self.arena, 0, global_ids=self.gids,
                             block_ids=ids_dev, block_size=B, block_dst=self.spare * B)
            self.ev_side.record(self.side)
            if self.phase_ms is not None:
                s1 = torch.cuda.Event(enable_timing=True)
                s1.record()
                self._side_events = (s0, s1)
        if pending is not None and len(wb_ids):
            _ops.dirty_mark(self.bitmap, wb_ids, False)
        self._phase("side_issue")
        self.plan_ahead(k)
        _ops.dirty_mark(self.bitmap, self.arena_block[slots].tolist(), True)
        _ops.block_bounds(self.arena["xyz"], (slots * B).tolist(), [B] * slots.size,
                          self.bounds[: slots.size])
        self.ev_main.record(main)
        self._phase("dirty_bounds")
        if dirty is not None:
            _ops.dirty_mark(self.bitmap, evicted_blocks[dirty].tolist(), True)
            _ops.dirty_mark(self.bitmap, evicted_blocks[~dirty].tolist(), False)
        order = np.argsort(evicted_blocks, kind="stable")
        self._pending_wb = (_ops.dirty_select_async(self.bitmap, evicted_blocks[order].tolist()),
                            evicted_blocks[order], evict_slots[order])
        self._phase("dirty_select")
        self._turn_over(k, evict_pos, incoming)
        self._phase("tables")
        return int(ids.numel())

    def drain(self) -> None:
        """Makes the current stream wait for the side stream's last work
        (the end of a timed region must cover it)."""
        if self.overlap:
            torch.cuda.current_stream(self.device).wait_event(self.ev_side)

    _side_events = None
    param_gather = None

    def close(self):
        """Releases the peer mappings (collective over the ranks)."""
        for attr in ("peer", "pull", "param_gather"):
            obj = getattr(self, attr)
            if obj is not None:
                obj.close()
                setattr(self, attr, None)

    def parity_check(self, k: int, blocks_per_owner: int = 2, rows: int = 256) -> dict:
        """Checker, run after the timed region (not part of any measured
        number): step k runs as usual while sampled rows of `blocks_per_owner`
        of each owner's updated blocks are replayed on the CPU through the
        kernel-order Adam restatement (oracle/resident_adam.py, pinned to the
        reference's update, gpu_resident_optimizer.py:339-364) on the
        rank-order sum of every rank's gradient contribution to the block.
        Parameters, both moments and the row stamps must match bit for bit.
        A row's update depends only on its own values and its slot's step, so
        a window of `rows` rows of a block stands for the block. Every rank
        takes the same collective steps (two object all-gathers and a final
        one for the counts)."""
        from oracle.resident_adam import bias_pair, kernel_update

        torch.cuda.synchronize()  # the side stream's blocks of the last step have landed
        W, me, sched = self.world, self.sched.rank, self.sched
        pos_all = sched.visible_positions(k)
        evict_pos = self.trace.turn[k][0]
        rng = np.random.default_rng(777 + 31 * k + me)
        # positions whose parameters survive the step (evicted slots are
        # overwritten by the incoming blocks at its end)
        cand = np.setdiff1d(pos_all, evict_pos)
        pick = np.sort(rng.choice(cand, min(blocks_per_owner, cand.size), replace=False))
        # (block, its arena slot, first row of the window)
        mine = [(int(sched.slot_block[p]), int(self.arena_of_pos[p]),
                 int(rng.integers(0, B - rows + 1))) for p in pick]
        vis_slots = self.visible_arena(k)

        def gather(obj):
            if W == 1:
                return [obj]
            import torch.distributed as dist

            out = [None] * W
            dist.all_gather_object(out, obj)
            return out

        samples = gather(mine)  # [owner] -> [(block, arena slot, first row)]
        # this rank's gradient rows for every sampled block it rendered
        contrib = {}
        if W == 1:
            for b, p, r0 in mine:
                i = int(np.searchsorted(vis_slots, p))
                contrib[(0, b)] = np.concatenate(
                    [self.grads[n][i * B + r0: i * B + r0 + rows].cpu().numpy()
                     for n in NAMES], axis=1)
        else:
            rendered = np.unique(self.trace.vis[k][me])
            for o, lst in enumerate(samples):
                for b, _, r0 in lst:
                    j = int(np.searchsorted(rendered, b))
                    if j < rendered.size and rendered[j] == b:
                        contrib[(o, b)] = np.concatenate(
                            [self.rank_grads[n][j * B + r0: j * B + r0 + rows].cpu().numpy()
                             for n in NAMES], axis=1)
        by_rank = gather(contrib)
        # snapshot of the owner's rows before the step
        before = []
        for b, p, r0 in mine:
            lo = p * B + r0
            before.append(dict(
                params={n: self.arena[n][lo:lo + rows].cpu().numpy() for n in NAMES},
                state=self.state[lo:lo + rows].cpu().numpy(),
                step=int(self.slot_step[p].item()), stamp=int(self.stamp_host[p])))
        self.step(k)
        torch.cuda.synchronize()
        checked = mismatched = 0
        for (b, p, r0), snap in zip(mine, before):
            parts = [d[(me, b)] for d in by_rank if (me, b) in d]  # rank order
            g = parts[0].copy()
            for x in parts[1:]:
                g = (g + x).astype(np.float32)
            st = snap["state"]
            fresh = st[:, 124].view(np.uint32) == np.uint32(snap["stamp"])
            m0 = np.where(fresh[:, None], st[:, 0:118:2], np.float32(0))
            v0 = np.where(fresh[:, None], st[:, 1:118:2], np.float32(0))
            bias1, dscale = bias_pair(0.9, 0.999, snap["step"] + 1)
            lo = p * B + r0
            after_state = self.state[lo:lo + rows].cpu().numpy()
            ok = bool(np.all(after_state[:, 124].view(np.uint32) == np.uint32(snap["stamp"])))
            col = 0
            for n in NAMES:
                w = WIDTHS[n]
                pn, mn, vn = kernel_update(snap["params"][n], g[:, col:col + w],
                                           m0[:, col:col + w], v0[:, col:col + w], LRS[n],
                                           bias1, dscale, 0.9, 0.999, 1e-15, 16)
                got_p = self.arena[n][lo:lo + rows].cpu().numpy()
                ok &= np.array_equal(got_p.view(np.uint32), pn.view(np.uint32))
                ok &= np.array_equal(after_state[:, 2 * col:2 * (col + w):2].view(np.uint32),
                                     mn.view(np.uint32))
                ok &= np.array_equal(after_state[:, 2 * col + 1:2 * (col + w):2].view(np.uint32),
                                     vn.view(np.uint32))
                col += w
            checked += 1
            mismatched += 0 if ok else 1
        counts = gather((checked, mismatched, sum(len(v) for v in by_rank)))
        return {"checked_blocks": sum(c for c, _, _ in counts),
                "rows_per_block": rows, "step": k,
                "mismatched_blocks": sum(m for _, m, _ in counts),
                "bit_exact": all(m == 0 for _, m, _ in counts),
                "contributions": sum(c for _, _, c in counts) // max(1, W),
                "oracle": "oracle/resident_adam.py kernel_update on the rank-order sum of "
                          "the contributions (CPU, after the timed region)"}

    def measure_param_gather(self, k: int, iters: int = 10, warmup: int = 2,
                             sample: int = 2, rows: int = 256) -> dict:
        """Time, after the timed region, how long the parameters updated in
        step k-1 take to reach the ranks that render them in step k: each
        rank copies every block it renders at step k that another rank owns
        from the owner's arena (PeerParamGather: barrier, one bulk-copy
        launch per owner over NVLink, barrier). Blocks a rank owns are read
        in place. Then `sample` gathered blocks per rank are compared bit for
        bit with their owner's rows. Collective: every rank calls it."""
        import torch.distributed as dist

        from tidegs_b200.sharded import exchange_arena_tables, make_gather_plan

        W, me = self.world, self.sched.rank
        tables = exchange_arena_tables(self.arena_block, self.device)
        plan = make_gather_plan(self.trace.vis[k][me], tables, W, me, B)
        n = int(plan.remote_blocks.size)
        render = {nm: torch.empty((max(1, n) * B, w), device=self.device)
                  for nm, w in WIDTHS.items()}
        dev_tables = self.param_gather.tables(plan)
        for _ in range(warmup):
            self.param_gather.gather(render, plan, dev_tables, err=self.err)
        torch.cuda.synchronize()
        copy_ev, full_ev = [], []
        for _ in range(iters):
            f0, c0, c1, f1 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
            f0.record()
            self.param_gather.barrier()
            c0.record()
            self.param_gather.launch(render, plan, dev_tables, err=self.err)
            c1.record()
            self.param_gather.barrier()
            f1.record()
            copy_ev.append((c0, c1))
            full_ev.append((f0, f1))
        torch.cuda.synchronize()
        copy_ms = sum(a.elapsed_time(b) for a, b in copy_ev) / iters
        full_ms = sum(a.elapsed_time(b) for a, b in full_ev) / iters
        # bit-exact check of sampled blocks against their owners' rows
        rng = np.random.default_rng(99 + me)
        pick = np.sort(rng.choice(n, min(sample, n), replace=False)) if n else np.zeros(0, int)
        asks = [(int(plan.owner[i]), int(plan.src_slot[i]),
                 int(rng.integers(0, B - rows + 1))) for i in pick]
        got = [np.concatenate([render[nm][i * B + r0:i * B + r0 + rows].cpu().numpy()
                               for nm in NAMES], axis=1) for i, (_, _, r0) in zip(pick, asks)]
        all_asks = [None] * W
        dist.all_gather_object(all_asks, asks)
        answers = {}
        for r, lst in enumerate(all_asks):
            for j, (o, slot, r0) in enumerate(lst):
                if o == me:
                    lo = slot * B + r0
                    answers[(r, j)] = np.concatenate(
                        [self.arena[nm][lo:lo + rows].cpu().numpy() for nm in NAMES], axis=1)
        all_answers = [None] * W
        dist.all_gather_object(all_answers, answers)
        ok = True
        for j, g in enumerate(got):
            want = next(a[(me, j)] for a in all_answers if (me, j) in a)
            ok = ok and np.array_equal(g.view(np.uint32), want.view(np.uint32))
        del render
        per_rank = [None] * W
        dist.all_gather_object(per_rank, (n, copy_ms, full_ms, len(got), bool(ok),
                                          int(plan.missing.size)))
        nbytes = max(x[0] for x in per_rank) * B * 59 * 4
        copy_max = max(x[1] for x in per_rank)
        return {"step": k, "iters": iters,
                "remote_blocks_per_rank": [x[0] for x in per_rank],
                "bytes_per_rank_max": nbytes,
                "copy_ms_max_over_ranks": copy_max,
                "with_barriers_ms_max_over_ranks": max(x[2] for x in per_rank),
                "GBps_per_rank": nbytes / (copy_max / 1e3) / 1e9,
                "nvlink_frac": nbytes / (copy_max / 1e3) / 1e9 / NVLINK_GBPS,
                "nvlink_peak_GBps": NVLINK_GBPS,
                "missing_blocks": sum(x[5] for x in per_rank),
                "checked_blocks": sum(x[3] for x in per_rank),
                "bit_exact": all(x[4] for x in per_rank),
                "how": "PeerParamGather: every block a rank renders next and another rank "
                       "owns, copied whole from the owner's arena slot over NVLink "
                       "(tgs_copy_blocks, bulk copies, one launch per owner); not part of "
                       "the timed step"}

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

    def __init__(self, device, sched: "Schedule", trace: ScheduleTrace, rank: int, world: int,
                 pool_blocks: int, host_blocks: np.ndarray, exchange: str = "pull",
                 host_tier: str = "cache"):
        import types

        from tidegs_b200 import (BlockLayout, CachedBlockReader, DoubleBufferGPUWorkingSet,
                                 GPUResidentAdam, GPUWorkingSet, PinnedBlockCache,
                                 PinnedBlockPool, _ops)

        self.device = device
        self.trace = trace
        self.sched = sched
        self.rank, self.world = rank, world
        num_total = SCENE_BLOCKS * B
        gen = torch.Generator().manual_seed(99 + rank)
        self.cache = None
        self.host_blocks = np.asarray(host_blocks, np.int64)
        if host_tier == "cache":
            # the host tier holds every block this rank touches in the timed
            # steps (host_blocks): pool_blocks distinct seeded blocks, scene
            # block b holding distinct[b % pool_blocks], read into the cache's
            # page-locked slab through its prefetch; room for one write-back
            # batch of fresh entries on top
            distinct = torch.empty((pool_blocks, B, 59))
            for i in range(pool_blocks):
                distinct[i].normal_(0.0, 1.0, generator=gen)
            store = _SceneStore(distinct)
            self.cache = PinnedBlockCache(store, max_ram_gb=1e9, block_size=B, verbose=False,
                                          capacity_blocks=self.host_blocks.size + TURNOVER)
            self.cache.prefetch(self.host_blocks.tolist())
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
        # the step's row ids: all rows of the visible positions, uploaded as
        # positions from page-locked memory and expanded on the device
        max_rows = sched.traj.max_owned_visible() * B
        self.pos_pinned = torch.empty(2 * (max_rows // B), dtype=torch.int64).pin_memory()
        self.ids_buf = torch.empty(max_rows, dtype=torch.int64, device=device)
        self.grads = {n: torch.empty((max_rows, w), device=device).normal_(0, 1e-3)
                      for n, w in WIDTHS.items()}
        self.peer = None
        self.pull = None
        if world > 1:
            send_max, recv_max = exchange_capacity(sched, world, trace.n_steps)
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
        pos = self.sched.visible_positions(k)
        if self.world == 1:
            ids = self._row_ids(pos, k)
            return ids, {name: g[:ids.numel()] for name, g in self.grads.items()}
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
        slices = self.db.active_buffer.block_to_local_slice
        probe = plan.out_blocks[:: max(1, plan.n_out // 16)]
        if (not np.array_equal(slot_of[plan.out_blocks], pos)
                or any(slices[int(b)].start != slot_of[int(b)] * B for b in probe)):
            raise RuntimeError("exchange plan and owner slices disagree")
        return self._row_ids(pos, k), grads

    def _row_ids(self, pos: np.ndarray, k: int) -> torch.Tensor:
        """All rows of the visible slot positions: the positions go up from
        page-locked memory (counted as H2D bytes), the rows are expanded on
        the device. Two host buffers alternate by step."""
        from tidegs_b200 import _ops

        half = self.pos_pinned.numel() // 2
        if pos.size > half:
            raise RuntimeError(f"{pos.size} visible positions exceed the position buffer")
        host = self.pos_pinned[(k % 2) * half:(k % 2) * half + pos.size]
        host.numpy()[:] = pos
        self.h2d_bytes += pos.size * 8
        dev_pos = self._upload_ids(host)
        n = int(pos.size) * B
        ids = self.ids_buf[:n]
        _ops.fill_global_ids(ids, 0, dev_pos, n, B)
        return ids

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

    def step(self, k: int, turn=None, optimize: bool = True) -> int:
        """One iteration in the engine's order: the resident plan for k+1 is
        known up front and its N+1 prefetch (H2D of the incoming blocks) runs
        on the worker thread / prefetch stream while the optimizer step and
        the write-back of iteration k run. `turn` overrides the trace's
        turnover (evicted positions, incoming blocks, dirty pattern or None);
        optimize=False leaves out the optimizer and the bounds
        (materialization only, configs[2]), marking the evicted blocks dirty
        by the pattern instead."""
        db, ws, sched = self.db, self.ws, self.sched
        t = time.perf_counter()
        if self.profile is not None:
            step_ev = torch.cuda.Event(enable_timing=True)
            step_ev.record()
            db.prefetch_events = {}
        evict_pos, incoming_arr, dirty = turn if turn is not None else self.trace.turn[k]
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
            if optimize:
                self.opt.set_resident_blocks(db.active_buffer.loaded_blocks)
            self._pending_activate = False
            t = self._mark("activate", t)
        rows = 0
        bounds = None
        if optimize:
            ids, grads = self._grads_and_ids(k)
            rows = int(ids.numel())
            t = self._mark("exchange", t)
            if isinstance(grads, tuple):
                stats = self.opt.step_pulled(k, self.gaussians, ids, *grads)
            else:
                stats = self.opt.step(k, self.gaussians, ids, grads)
            t = self._mark("adam_step", t)
            updated = stats["updated_block_ids"]
            db.mark_dirty_blocks(updated)
            bounds = ws.stage_block_bounds(updated)
        if dirty is not None:
            evicted_now = sched.slot_block[evict_pos]
            db.mark_dirty_blocks(evicted_now[dirty].tolist())
            db.mark_blocks_written_back(evicted_now[~dirty].tolist())
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
        self.h2d_bytes += len(incoming) * B * 59 * 4
        return rows


# ---------------------------------------------------------------------------
# The other configs of BASELINE.json, measured at N = 1 beside the step
# ---------------------------------------------------------------------------
def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def bench_selective_adam(device, steps: int = 10, warmup: int = 3) -> dict:
    """SelectiveAdam (optimizer.py:46-87 drop-in, one
    tgs_selective_adam launch for the six groups) over N = 1,048,576
    Gaussians, Bernoulli(0.3) visibility, grads N(0, 1e-3) on visible rows,
    10 steps from zero moments. Inputs (990 MB) exceed L2."""
    from tidegs_b200 import SelectiveAdam

    N = 1 << 20
    gen = torch.Generator(device=device).manual_seed(0)
    comps = {n: torch.empty((N, w), device=device) for n, w in WIDTHS.items()}
    fill_params(comps, gen)
    vis = torch.rand(N, generator=gen, device=device) < 0.3
    params = []
    for n in NAMES:
        p = torch.nn.Parameter(comps[n])
        p.grad = torch.randn(p.shape, generator=gen, device=device).mul_(1e-3) * vis[:, None]
        params.append(p)
    opt = SelectiveAdam([{"params": [p], "lr": LRS[n]} for p, n in zip(params, NAMES)],
                        eps=1e-15, betas=(0.9, 0.999))
    for _ in range(warmup):
        opt.step(vis)
    for p in params:
        opt.state[p]["exp_avg"].zero_()
        opt.state[p]["exp_avg_sq"].zero_()
    torch.cuda.synchronize()
    e0, e1 = _events()
    e0.record()
    for _ in range(steps):
        opt.step(vis)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    rows = int(vis.sum().item())
    nbytes = rows * 59 * 4 * 7 + N  # g r, p r/w, m r/w, v r/w per visible element; mask
    peak, kind = measured_peak()
    achieved = nbytes / (ms / 1e3) / 1e9
    return {"config": "configs[0]: SelectiveAdam, N=1,048,576 x 59, Bernoulli(0.3) rows, "
                      f"{steps} steps", "value": rows / (ms / 1e3), "unit": UNIT,
            "ms_per_step": ms, "visible_rows": rows,
            "roofline": {"bound": "hbm", "kernel": "dense_kernel<adam>", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": kind,
                         "algorithmic_bytes": "28 B per visible element + 1 B mask per row"}}


def bench_sophia(device, steps: int = 50, k: int = 10, warmup: int = 3) -> dict:
    """SelectiveSophia over N = 8,388,608 Gaussians, b1 0.965,
    b2 0.99, rho 0.04, Hessian EMA refreshed every k = 10 steps from a
    seeded N(0, 1) noise input, Bernoulli(0.3) visibility, 50 steps."""
    from tidegs_b200 import SelectiveSophia

    N = 8 * (1 << 20)
    gen = torch.Generator(device=device).manual_seed(1)
    comps = {n: torch.empty((N, w), device=device) for n, w in WIDTHS.items()}
    fill_params(comps, gen)
    vis = torch.rand(N, generator=gen, device=device) < 0.3
    params = []
    for n in NAMES:
        p = torch.nn.Parameter(comps[n])
        p.grad = torch.randn(p.shape, generator=gen, device=device).mul_(1e-3) * vis[:, None]
        params.append(p)
    noise = [torch.randn(p.shape, generator=gen, device=device) for p in params]
    groups = [{"params": [p], "lr": LRS[n]} for p, n in zip(params, NAMES)]
    opt = SelectiveSophia(groups, betas=(0.965, 0.99), rho=0.04, eps=1e-15, k=k)
    for _ in range(warmup):
        opt.step(vis, noise=noise)
    for p in params:
        st = opt.state[p]
        st["step"] = 0
        st["exp_avg"].zero_()
        st["hessian"].zero_()
    torch.cuda.synchronize()
    e0, e1 = _events()
    e0.record()
    for _ in range(steps):
        opt.step(vis, noise=noise)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    rows = int(vis.sum().item())
    hess_steps = sum(1 for t in range(1, steps + 1) if t % k == 1 % k)
    per_elem = (24 * steps + 8 * hess_steps) / steps
    nbytes = rows * 59 * per_elem + N
    peak, kind = measured_peak()
    achieved = nbytes / (ms / 1e3) / 1e9
    return {"config": f"configs[1]: SelectiveSophia, N=8,388,608 x 59, Bernoulli(0.3) rows, "
                      f"{steps} steps, Hessian every {k}", "value": rows / (ms / 1e3),
            "unit": UNIT, "ms_per_step": ms, "visible_rows": rows, "hessian_steps": hess_steps,
            "parity": "unpinned (the reference has no Sophia)",
            "roofline": {"bound": "hbm", "kernel": "dense_kernel<sophia>", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": kind,
                         "algorithmic_bytes": "24 B per visible element, +8 on Hessian steps, "
                                              "+1 B mask per row"}}


def link_probe(api, device, blocks_in: int, blocks_out: int) -> dict:
    """Host-link ceiling of this box: one DMA per block between page-locked
    host-cache entries and device memory, H2D alone, D2H alone, then both at
    once on two streams (the materialization's traffic pattern)."""
    from tidegs_b200 import _ops

    slab = api.cache.slab if api.cache is not None else None
    if slab is None:
        return {"skipped": "no page-locked host cache"}
    nb = min(blocks_in, slab.shape[0] // 2)
    no = min(blocks_out, slab.shape[0] - nb)
    dev = torch.empty((max(nb, no), B, 59), device=device)
    bpb = B * 59 * 4
    h_src = [slab[i].data_ptr() for i in range(nb)]
    h_dst = [dev[i].data_ptr() for i in range(nb)]
    d_src = [dev[i].data_ptr() for i in range(no)]
    d_dst = [slab[nb + i].data_ptr() for i in range(no)]
    side = torch.cuda.Stream(device)

    def run(h2d, d2h):
        torch.cuda.synchronize()
        a0, a1 = _events()
        b0, b1 = _events()
        a0.record()
        if h2d:
            _ops.h2d_blocks(h_dst, h_src, [bpb] * nb, device)
        a1.record()
        with torch.cuda.stream(side):
            b0.record(side)
            if d2h:
                _ops.d2h_blocks(d_dst, d_src, [bpb] * no, device)
            b1.record(side)
        torch.cuda.synchronize()
        return a0.elapsed_time(a1), b0.elapsed_time(b1)

    run(True, True)
    h_ms, _ = run(True, False)
    _, d_ms = run(False, True)
    hc_ms, dc_ms = run(True, True)
    del dev
    return {"h2d_GBps": nb * bpb / h_ms / 1e6, "d2h_GBps": no * bpb / d_ms / 1e6,
            "concurrent_h2d_GBps": nb * bpb / hc_ms / 1e6,
            "concurrent_d2h_GBps": no * bpb / dc_ms / 1e6,
            "concurrent_total_GBps": (nb + no) * bpb / max(hc_ms, dc_ms) / 1e6,
            "blocks": [nb, no]}


def bench_materialization(api, device, first_k: int, iterations: int = 240,
                          warmup: int = 3) -> dict:
    """materialization only over the e2e leg's host tier: each
    iteration TURNOVER random slots take random non-resident blocks of the
    rank's page-locked host cache (random block-id -> slot remap; H2D,
    unpack, slot swap through DoubleBufferGPUWorkingSet), Bernoulli(0.5)
    dirty flags on the evicted blocks, compacted and written back into the
    cache (GPUWorkingSet.stage_updated_blocks, D2H)."""
    turn = RandomTurnover(api.sched.slot_block, api.host_blocks, seed=3)
    for i in range(warmup):
        api.step(first_k + i, turn=turn.turnover(i), optimize=False)
    torch.cuda.synchronize()
    api.h2d_bytes = api.d2h_bytes = 0
    e0, e1 = _events()
    t0 = time.perf_counter()
    e0.record()
    for i in range(warmup, warmup + iterations):
        api.step(first_k + i, turn=turn.turnover(i), optimize=False)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = e0.elapsed_time(e1)
    link = link_probe(api, device, TURNOVER, TURNOVER // 2)
    moved = api.h2d_bytes + api.d2h_bytes
    achieved = moved / (ms / 1e3) / 1e9
    ceiling = link.get("concurrent_total_GBps")
    return {"config": f"configs[2]: {SLOTS} slots x {B}, {TURNOVER} random slots replaced per "
                      f"iteration from the rank's page-locked host tier "
                      f"({api.host_blocks.size} blocks), Bernoulli(0.5) dirty write-back, "
                      f"{iterations} iterations",
            "ms_per_iteration": ms / iterations, "wall_ms_per_iteration": 1e3 * wall / iterations,
            "h2d_bytes_per_iteration": api.h2d_bytes / iterations,
            "d2h_bytes_per_iteration": api.d2h_bytes / iterations,
            "host_link_GBps": achieved, "link_ceiling": link,
            "frac_of_link_ceiling": (achieved / ceiling) if ceiling else None}


# ---------------------------------------------------------------------------
# CPU baseline and reference arm: the reference's torch CPU path of the same
# step (oracle/cpu_step.py), on the same seeded schedule
# ---------------------------------------------------------------------------
def run_cpu_step(slots: int, steps: int, warmup: int, seconds_budget: float = None) -> dict:
    """Runs the reference's CPU step over `slots` resident slots (the
    workload's other ratios kept) on this workload's schedule: `warmup`
    untimed steps, then `steps` timed ones (or, with a budget, as many as fit
    in `seconds_budget`, at least one). All host threads."""
    from oracle.cpu_step import ReferenceCpuStep

    # The CPU step allocates its temporaries (index_select results, ~0.2 GB
    # each) anew every step, as the reference does. Keep freed heap memory
    # for reuse instead of returning it to the kernel, so that the baseline
    # is not charged a fresh round of page faults per step.
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6")
        libc.mallopt(-3, ctypes.c_int(2 ** 31 - 1))  # M_MMAP_THRESHOLD
        libc.mallopt(-1, ctypes.c_int(2 ** 31 - 1))  # M_TRIM_THRESHOLD
    except OSError:
        pass
    saved = SLOTS
    set_slots(slots)
    try:
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        n_trace = warmup + (steps if seconds_budget is None else 10_000) + 1
        sched = Schedule(0, 1)
        max_vis = sched.traj.max_owned_visible() * B
        cpu = ReferenceCpuStep(SLOTS, B, TURNOVER, max_vis, pool_blocks=32,
                               num_blocks=SCENE_BLOCKS, seed=0)
        rows_in_block = torch.arange(B, dtype=torch.int64)

        def one(k):
            pos = sched.visible_positions(k)
            # the touched rows, as the engine lists them (all rows of the
            # visible blocks, ascending)
            ids = (torch.from_numpy(pos)[:, None] * B + rows_in_block[None, :]).reshape(-1)
            evict_pos, incoming, dirty = sched.turnover(k)
            n = cpu.step(ids, sched.slot_block[pos].tolist(), pos, evict_pos,
                         sched.slot_block[evict_pos].copy(), incoming, dirty)
            sched.slot_block[evict_pos] = incoming
            return n

        for k in range(warmup):
            one(k)
        rows = done = 0
        t0 = time.perf_counter()
        k = warmup
        while k < n_trace - 1:
            rows += one(k)
            done += 1
            k += 1
            if seconds_budget is None:
                if done == steps:
                    break
            elif time.perf_counter() - t0 > seconds_budget:
                break
        elapsed = time.perf_counter() - t0
        return {"value": rows / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
                "ms_per_step": 1e3 * elapsed / done, "steps": done, "warmup": warmup,
                "slots": SLOTS, "rows_per_step": rows / done,
                "sample": (f"{SLOTS} slots x {B} rows ({'a full GPU resident set' if SLOTS == 2048 else f'{SLOTS}/2048 of a GPU resident set'}), "
                           f"the bench's schedule at one rank (~30% of the slots visible, all "
                           f"their rows updated; {TURNOVER} blocks turned over, dirty ones "
                           f"written back), "
                           f"{done} timed steps after {warmup} warm-up steps in {elapsed:.1f} s: "
                           "the reference's torch CPU step (oracle/cpu_step.py: optimizer "
                           "gpu_resident_optimizer.py:266-364, dirty marks, bounds, write-back "
                           "pack gpu_working_set.py:968-975, block staging, unpack, id fill and "
                           "slot swap double_buffer_gpu.py:791-837,944-951,1053-1062, moments "
                           "cleared on admission)")}
    finally:
        set_slots(saved)


def cpu_baseline(seconds_budget: float = 15.0):
    """The cpu_baseline object of this arm's line: a bounded sample (64 of
    the 2048 slots, the same ratios) for about `seconds_budget` seconds."""
    base = run_cpu_step(64, 0, 2, seconds_budget=seconds_budget)
    return {k: base[k] for k in ("value", "unit", "cores", "kind", "sample", "ms_per_step")}


def reference_arm_slots(limit: int) -> int:
    """Resident slots the reference arm can hold in this host's memory: the
    full 2048 when the CPU step's buffers fit in 70 % of it, else halved
    until they do."""
    from oracle.cpu_step import host_bytes

    slots = SLOTS
    while slots > 64 and host_bytes(slots, B, max(1, slots // 4), 0.35, 32) > 0.7 * limit:
        slots //= 2
    return slots


def run_reference_arm(args, world, rank):
    """`--impl reference`: the reference's own CPU implementation of the
    step, the whole configs[3] workload when the host holds it (else the
    largest power-of-two share that fits, stated), timed over exactly
    --steps steps after --warmup steps, on rank 0 (other ranks exit)."""
    if rank != 0:
        return 0
    slots = reference_arm_slots(host_memory_limit())
    # keep the whole run to a few minutes: a short calibration on a small
    # share gives this host's rate; halve the share until the run's
    # --steps + --warmup steps are expected to take under 150 s (the rate
    # drops on larger working sets, hence the margin)
    rate = run_cpu_step(64, 2, 1)["value"]
    rows_full = VISIBLE_FRAC * SLOTS * B
    while slots > 64 and (args.steps + args.warmup) * rows_full * (slots / SLOTS) / rate * 1.5 > 150:
        slots //= 2
    base = run_cpu_step(slots, args.steps, args.warmup)
    same = slots == SLOTS
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": base["steps"], "warmup": base["warmup"],
        "ms_per_step": base["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE configs[3] shapes and distributions)",
        "config": dict(WORKLOAD_CONFIG, slots_per_gpu=slots, block_size=B,
                       turnover_blocks=max(1, slots // 4),
                       rows_updated_per_step=base["rows_per_step"],
                       run=("the reference's CPU step on this arm's full workload"
                            if same else
                            f"the reference's CPU step on {slots} of the workload's {SLOTS} "
                            "slots (to fit this host's memory and a run of a few minutes), same "
                            "ratios; value and ms_per_step are that sample's")
                       + ", all host threads, rank 0 only"),
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
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-warmup", type=int, default=4)
    ap.add_argument("--e2e-profile", action="store_true",
                    help="print a per-phase wall-time breakdown of the e2e step to stderr")
    ap.add_argument("--pool-blocks", type=int, default=256,
                    help="distinct seeded host blocks (scene block b holds block b mod this)")
    ap.add_argument("--host-tier", default="cache", choices=["cache", "pool"],
                    help="e2e host side: PinnedBlockCache over every block the rank touches "
                         "(write-back lands in it), or the fixed modulo PinnedBlockPool")
    ap.add_argument("--no-configs", action="store_true",
                    help="leave out the configs[0]/[1]/[2] measurements at N=1")
    ap.add_argument("--materialize-iters", type=int, default=240,
                    help="configs[2] iterations (materialization only)")
    ap.add_argument("--slots", type=int, default=SLOTS,
                    help="resident slots per GPU (default: the configs[3] value; smaller "
                         "values make small profiling cases of the same step)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--phase-times", action="store_true",
                    help="print a per-phase CUDA-event breakdown of the device step to stderr "
                         "(extra events; not used for the reported value)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--overlap", default="auto", choices=["auto", "on", "off"],
                    help="run the write-back and unpack on a side stream beside the update "
                         "(auto: on from OVERLAP_MIN_WORLD ranks, where NVLink bounds the "
                         "update and HBM has room)")
    ap.add_argument("--adam-ctas", type=int, default=-1,
                    help="cap on the streamed pull update's CTAs (-1: "
                         f"{OVERLAP_ADAM_CTAS} with --overlap, else one per SM)")
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

    from tidegs_b200 import _lib

    device = torch.device("cuda", torch.cuda.current_device())
    n_e2e = args.e2e_warmup + args.e2e_steps
    host_blocks = Schedule(rank, world).touched_blocks(n_e2e + 1)
    args.host_tier = plan_host_tier(world, args.host_tier, args.pool_blocks,
                                    host_blocks.size, host_memory_limit())
    n_trace = max(args.warmup + args.steps + 6, n_e2e + 1)
    trace = ScheduleTrace(world, rank, n_trace)
    sched = Schedule(rank, world)
    overlap = args.overlap == "on" or (args.overlap == "auto" and world >= OVERLAP_MIN_WORLD)
    adam_ctas = args.adam_ctas if args.adam_ctas >= 0 else (OVERLAP_ADAM_CTAS if overlap else 0)
    dev = DeviceStep(device, sched, trace, world=world, exchange=args.exchange, overlap=overlap,
                     adam_ctas=adam_ctas)
    # sampling starts before the warm-up so that nvidia-smi is running when
    # the (short) timed region starts
    clocks = ClockSampler(device)
    for k in range(args.warmup):
        dev.step(k)
    torch.cuda.synchronize()
    barrier(world)
    launches0 = _lib.launch_counter["kernels"]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    rows = 0
    for k in range(args.warmup, args.warmup + args.steps):
        rows += dev.step(k, timed=True)
    dev.drain()
    end.record()
    torch.cuda.synchronize()
    next_k = args.warmup + args.steps
    if args.phase_times:
        # separate, untimed pass: per-phase CUDA events around each stage
        dev.phase_ms, dev.host_ms = {}, {}
        for k in range(next_k, next_k + 3):
            dev.step(k)
            dev.collect_phases()
        next_k += 3
        print(f"rank {rank} device phase ms/step: " + json.dumps(
            {n: round(sum(v) / len(v), 3) for n, v in dev.phase_ms.items()})
            + " host ms/step: " + json.dumps(
            {n: round(sum(v) / len(v), 3) for n, v in dev.host_ms.items()}),
            file=sys.stderr, flush=True)
        dev.phase_ms = dev.host_ms = None
    barrier(world)
    clock_info = clocks.stop()
    launches = _lib.launch_counter["kernels"] - launches0
    # result check of the same step, outside the timed region
    parity = dev.parity_check(next_k)
    param_gather = dev.measure_param_gather(next_k + 1) if world > 1 else None
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
    configs = {}
    host_link = None
    try:
        if args.no_e2e:
            raise _Skipped("--no-e2e")
        api = ApiStep(device, Schedule(rank, world), trace, rank, world, args.pool_blocks,
                      host_blocks, exchange=args.exchange, host_tier=args.host_tier)
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
               "host_tier": (f"PinnedBlockCache of the {host_blocks.size} blocks the rank "
                             f"holds during the e2e steps (+{TURNOVER} write-back entries; "
                             f"scene block b's rows = seeded block b mod {args.pool_blocks}); "
                             "write-back DMA into it"
                             if args.host_tier == "cache" else
                             f"PinnedBlockPool of {args.pool_blocks} blocks (block id mod pool)")}
        if api.profile is not None and rank == 0:
            print("e2e phase wall ms/step: " + json.dumps(
                {k: round(v * 1e3 / args.e2e_steps, 2) for k, v in api.profile.items()})
                + " writeback staging bytes: "
                + str(api.ws.writeback_stats["pinned_staging_bytes"]),
                file=sys.stderr, flush=True)
        if world == 1 and not args.no_configs and args.host_tier == "cache":
            configs["materialization"] = bench_materialization(
                api, device, n_e2e, iterations=args.materialize_iters)
        elif world > 1 and args.host_tier == "cache":
            # the box's host link with every rank copying at once (the e2e
            # leg's H2D + D2H pattern, no compute): what the ranks share
            barrier(world)
            mine = link_probe(api, device, TURNOVER, TURNOVER)
            host_link = _gather_all(mine, world)
        api.close()
        del api
    except _Skipped as why:
        e2e = {"value": None, "unit": UNIT, "skipped": str(why)}
    except Exception as exc:  # report, never hide
        e2e = {"value": None, "unit": UNIT, "error": f"{type(exc).__name__}: {exc}"}

    torch.cuda.empty_cache()
    if world == 1 and not args.no_configs:
        for name, fn in (("selective_adam", bench_selective_adam), ("sophia", bench_sophia)):
            try:
                configs[name] = fn(device)
            except Exception as exc:  # report, never hide
                configs[name] = {"error": f"{type(exc).__name__}: {exc}"}
            torch.cuda.empty_cache()

    base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base = cpu_baseline()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, BASELINE configs[3]/[4] shapes and distributions)",
            "config": {**WORKLOAD_CONFIG,
                       "slots_per_gpu": SLOTS, "block_size": B, "turnover_blocks": TURNOVER,
                       "scene_blocks": SCENE_BLOCKS,
                       "host_tier_blocks_per_gpu": int(host_blocks.size),
                       "rows_updated_per_step": rows / args.steps,
                       "parallelism": f"block ownership, rank = block_id mod {world}",
                       "exchange_rows_per_step": exchange_rows / (args.warmup + args.steps),
                       "exchange": (None if world == 1 else
                                    "owner update kernel sums senders' gradients over NVLink "
                                    "(tgs_resident_adam_apply_sum)" if args.exchange == "pull"
                                    else "direct NVLink push (tgs_grad_push) + ordered owner sum"
                                    if args.exchange == "push" else
                                    "pack + NCCL all-to-all + ordered owner sum"),
                       "materialization": ("write-back of the previous step's evicted blocks "
                                           "and unpack on a side stream beside the update "
                                           f"(update capped at {adam_ctas} CTAs)" if overlap
                                           else "after the update, on the same stream"),
                       "l2": "every input larger than L2 (126 MB)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": ADAM_TRAFFIC_BYTES_PER_ROW * (sum(adam_rows) / len(adam_rows)),
                         "traffic_note": "bytes per launch: ncu DRAM bytes per row of the "
                                         "256-slot capture x rows per launch",
                         "kernel": "resident_adam_stream_kernel (+ resident_adam_kernel for "
                                   "chunks that cannot stream)",
                         "algorithmic_bytes_per_row": ADAM_BYTES_PER_ROW,
                         "avg_launch_ms": adam_avg_ms, "peak_source": peak_kind,
                         "avg_launch_ms_max_over_ranks": adam_max_ms},
            "clocks": clock_info,
            "gpu_launches": launches,
            "parity": parity,
            "param_gather": param_gather,
            "e2e": e2e,
            "cpu_baseline": base,
            "configs": configs or None,
        }
        if host_link is not None:
            line["host_link_all_ranks"] = {
                "per_rank_concurrent_GBps": [r.get("concurrent_total_GBps") for r in host_link],
                "box_total_GBps": sum(r.get("concurrent_total_GBps") or 0 for r in host_link),
                "probe": "every rank at once: one DMA per block, TURNOVER blocks H2D and "
                         "TURNOVER blocks D2H on two streams, page-locked host cache entries"}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
