"""Multi-GPU block ownership: gradient exchange to block owners.

TideGS itself is single-GPU. On a multi-GPU box the blocks shard by id
(owner rank = block_id mod world): each rank keeps resident slots and Adam
state only for the blocks it owns, renders its share of the camera batch, and
produces gradient tiles for every block its cameras saw, whoever owns it.
Before the owner's fused Adam step those tiles are reduced onto the owner:

  1. plan       every rank derives the same plan from the global schedule
                (which rank saw which blocks); no count exchange is needed;
  2. pack       the rank's gradient rows of each visible block are gathered
                into [block_size, 59] UNIFIED-order tiles, grouped by owner
                (tgs_pack_rows);
  3. exchange   one all-to-all with uneven splits (NCCL on GPUs; the same
                code runs on gloo for CPU tests), or, fused with step 2, a
                direct push: one kernel gathers each tile and stores it into
                the owner's receive buffer over NVLink (PeerGradExchange);
  4. reduce     the owner sums the tiles of each of its blocks in sender-rank
                order straight into the compact SoA gradients the resident
                Adam step consumes (tgs_block_grad_sum).

Because the summation order is fixed (rank 0 first), the owner's gradients
equal a single-GPU sum of all ranks' contributions in rank order bit for bit,
and so does the following Adam update.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Sequence

import numpy as np
import torch

from . import _lib, _ops


def owner_of(block_ids, world: int) -> np.ndarray:
    """Owning rank of each block id."""
    return np.asarray(block_ids, dtype=np.int64) % int(world)


@dataclass
class ExchangePlan:
    world: int
    rank: int
    block_size: int
    send_blocks: np.ndarray      # this rank's visible blocks, grouped by owner, ascending id
    send_counts: List[int]       # blocks sent to each owner
    recv_blocks: np.ndarray      # block id of each received tile (sender 0's tiles first)
    recv_counts: List[int]       # blocks received from each sender
    out_blocks: np.ndarray       # the owner's visible blocks, in output row order
    contrib_offsets: np.ndarray  # [n_out + 1] CSR offsets into contrib_blocks
    contrib_blocks: np.ndarray   # received tile index of each contribution, sender order
    send_dst_tiles: np.ndarray   # tile index of each sent block in its owner's receive rows
    recv_src_tiles: np.ndarray   # index of each received block among its sender's rendered
                                 # blocks (ascending id): its tile in the sender's gradients

    @property
    def n_out(self) -> int:
        return int(self.out_blocks.size)


def make_plan(visible_by_rank: Sequence[Sequence[int]], world: int, rank: int, block_size: int,
              out_order=None) -> ExchangePlan:
    """Builds this rank's send/receive plan.

    visible_by_rank[r] = blocks whose gradients rank r produced this step.
    out_order (optional) maps each owned block to its sort key in the owner's
    gradient rows (for example the start row of its resident slice, so that
    the owner's local row ids come out ascending); default: block id. It is a
    mapping, or a dense int64 table indexed by block id whose negative
    entries mark blocks without a position.
    """
    world = int(world)
    if len(visible_by_rank) != world:
        raise ValueError(f"visible_by_rank has {len(visible_by_rank)} entries for world={world}")
    vis = [np.unique(np.asarray(v, dtype=np.int64)) for v in visible_by_rank]
    for v in vis:
        if v.size and v[0] < 0:
            raise ValueError("block ids must be non-negative")
    mine = vis[rank]
    own = owner_of(mine, world)
    order = np.lexsort((mine, own))
    send_blocks = mine[order]
    send_counts = np.bincount(own, minlength=world).astype(np.int64).tolist()
    # where an all-to-all would put each sent tile on its owner: after the
    # tiles of lower senders for that owner, in ascending block order
    before = np.zeros(world, np.int64)
    for r in range(rank):
        before += np.bincount(owner_of(vis[r], world), minlength=world)
    group_start = np.concatenate([[0], np.cumsum(send_counts)[:-1]]).astype(np.int64)
    send_owner = own[order]
    send_dst_tiles = (before[send_owner] + np.arange(send_blocks.size, dtype=np.int64)
                      - group_start[send_owner])
    recv_lists = [v[owner_of(v, world) == rank] for v in vis]
    recv_counts = [int(x.size) for x in recv_lists]
    recv_blocks = (np.concatenate(recv_lists) if recv_lists else np.zeros(0, np.int64))
    recv_src_tiles = np.concatenate([np.nonzero(owner_of(v, world) == rank)[0] for v in vis]
                                    ).astype(np.int64)
    # group received tiles by block; a stable sort keeps sender order inside a block
    idx = np.argsort(recv_blocks, kind="stable")
    sorted_ids = recv_blocks[idx]
    uniq, first = np.unique(sorted_ids, return_index=True)
    counts = np.diff(np.append(first, sorted_ids.size))
    if out_order is not None:
        keys = _order_keys(out_order, uniq)
        perm = np.argsort(keys, kind="stable")
    else:
        perm = np.arange(uniq.size)
    out_blocks = uniq[perm]
    lens = counts[perm].astype(np.int64)
    offsets = np.zeros(uniq.size + 1, np.int64)
    np.cumsum(lens, out=offsets[1:])
    # contributions of out block k: idx[first[perm[k]] : + lens[k]], concatenated
    within = np.arange(int(offsets[-1]), dtype=np.int64) - np.repeat(offsets[:-1], lens)
    contrib = idx[np.repeat(first[perm].astype(np.int64), lens) + within]
    return ExchangePlan(world, rank, int(block_size), send_blocks, send_counts, recv_blocks,
                        recv_counts, out_blocks, offsets, contrib.astype(np.int64),
                        send_dst_tiles, recv_src_tiles)


def _order_keys(out_order, blocks: np.ndarray) -> np.ndarray:
    """Sort keys of `blocks` from a mapping or a dense table (block id ->
    key, negative = block not owned here)."""
    if isinstance(out_order, np.ndarray):
        inside = blocks < out_order.size
        keys = np.full(blocks.size, -1, np.int64)
        keys[inside] = out_order[blocks[inside]]
        missing = blocks[keys < 0]
    else:
        missing = np.asarray([int(b) for b in blocks if int(b) not in out_order], np.int64)
        keys = (np.asarray([out_order[int(b)] for b in blocks], dtype=np.int64)
                if missing.size == 0 else None)
    if missing.size:
        raise KeyError(f"blocks {missing[:8].tolist()} have no position in the owner's rows")
    return keys


def _send_starts(plan: ExchangePlan, block_row_start) -> np.ndarray:
    """First compact gradient row of each sent block: block_row_start is a
    mapping block -> row, or an int64 array aligned with plan.send_blocks."""
    if isinstance(block_row_start, np.ndarray):
        starts = np.asarray(block_row_start, np.int64)
        if starts.shape != plan.send_blocks.shape:
            raise ValueError("block_row_start array must align with plan.send_blocks")
        return starts
    return np.asarray([int(block_row_start[int(b)]) for b in plan.send_blocks], np.int64)


def _sum_tiles(plan: ExchangePlan, recv_ptr: int, device: torch.device,
               out: Optional[Mapping[str, torch.Tensor]], err: Optional[torch.Tensor]
               ) -> Dict[str, torch.Tensor]:
    """Owner-side ordered sum of the received tiles (tgs_block_grad_sum)."""
    B = plan.block_size
    rows = plan.n_out * B
    if out is None:
        out = {n: torch.empty((rows, w), dtype=torch.float32, device=device)
               for n, w in _ops.WIDTHS.items()}
    else:
        out = {n: t[:rows] for n, t in out.items()}
    if plan.n_out == 0:
        return out
    tables = _ops.i64_to_device(np.concatenate([plan.contrib_offsets, plan.contrib_blocks]),
                                device)
    args = _lib.BlockSumArgs()
    args.recv = recv_ptr
    args.n_recv_blocks = int(sum(plan.recv_counts))
    args.contrib_offsets = tables.data_ptr()
    args.contrib_blocks = tables[plan.n_out + 1:].data_ptr()
    args.n_out = plan.n_out
    args.block_size = B
    for c, name in enumerate(_ops.COMPONENTS):
        args.out[c] = out[name].data_ptr()
    args.err = _lib.ptr(err)
    _lib.call("tgs_block_grad_sum", args, _lib.stream_handle(device))
    tables.record_stream(torch.cuda.current_stream(device))
    return out


class BlockGradExchange:
    """Runs a plan: pack -> all-to-all (NCCL) -> ordered sum on the owner."""

    def __init__(self, block_size: int, group=None, device: Optional[torch.device] = None):
        self.block_size = int(block_size)
        self.group = group
        self.device = device

    def pack(self, plan: ExchangePlan, grads: Mapping[str, torch.Tensor],
             block_row_start, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Gathers the rows of each sent block (block_row_start[b] = first
        row of block b in the compact gradient tensors, or an array aligned
        with plan.send_blocks) into UNIFIED tiles."""
        n = int(plan.send_blocks.size) * self.block_size
        dev = grads["xyz"].device
        if out is None:
            out = torch.empty((n, 59), dtype=torch.float32, device=dev)
        if n:
            starts = _send_starts(plan, block_row_start)
            refs = _ops.pack_rows(grads, starts, [self.block_size] * starts.size, out[:n],
                                  _lib.LAYOUT_UNIFIED)
            del refs
        return out[:n]

    def all_to_all(self, plan: ExchangePlan, send: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
        import torch.distributed as dist

        B = self.block_size
        n_recv = int(sum(plan.recv_counts)) * B
        recv = out[:n_recv] if out is not None else torch.empty(
            (n_recv, 59), dtype=send.dtype, device=send.device)
        if plan.world == 1:
            recv.copy_(send)
            return recv
        dist.all_to_all_single(recv, send, [c * B for c in plan.recv_counts],
                               [c * B for c in plan.send_counts], group=self.group)
        return recv

    def reduce(self, plan: ExchangePlan, recv: torch.Tensor,
               out: Optional[Mapping[str, torch.Tensor]] = None,
               err: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """Compact SoA gradients of the owner's visible blocks (plan.out_blocks
        order, block_size rows each)."""
        return _sum_tiles(plan, recv.data_ptr(), recv.device, out, err)


class PeerGradExchange:
    """Runs a plan with direct NVLink stores instead of pack + all-to-all.

    Every rank allocates `n_buffers` receive buffers of `capacity_blocks`
    UNIFIED tiles through tgs_peer_buffer_alloc and maps every other rank's
    buffers (CUDA IPC handles swapped with one all-gather). A step is

        push(plan, grads, starts, parity)   # tgs_grad_push into the owners' buffers
        barrier()                           # every rank's push has finished
        reduce(plan, parity, out)           # owner-side ordered sum (own buffer)

    all on the caller's current stream. The barrier is a one-element
    all-reduce: its completion on a rank means every rank launched it, i.e.
    finished its push. Consecutive steps alternate the buffer parity, so a
    push of step k+1 (issued after the barrier of step k) never overwrites
    tiles an owner still sums for step k-1. Tiles land exactly where the
    all-to-all of BlockGradExchange puts them, so both give identical sums.
    """

    def __init__(self, block_size: int, capacity_blocks: int, device, group=None,
                 n_buffers: int = 2):
        import ctypes

        import torch.distributed as dist

        self.device = _lib.require_cuda(device, "PeerGradExchange")
        self.block_size = int(block_size)
        self.capacity_rows = int(capacity_blocks) * self.block_size
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if self.world > _lib.MAX_PEERS:
            raise RuntimeError(f"PeerGradExchange supports at most {_lib.MAX_PEERS} ranks")
        self.n_buffers = int(n_buffers)
        lib = _lib.load()
        nbytes = max(self.capacity_rows, 1) * 59 * 4
        self._own: List[int] = []
        handles = bytearray()
        with torch.cuda.device(self.device):
            for _ in range(self.n_buffers):
                ptr = ctypes.c_void_p()
                h = _lib.PeerHandle()
                _lib.call("tgs_peer_buffer_alloc", nbytes, ctypes.byref(ptr), ctypes.byref(h))
                self._own.append(int(ptr.value))
                handles += bytes(h.bytes)
            # recv[parity][rank] = that rank's buffer as mapped here
            self.recv = [[0] * self.world for _ in range(self.n_buffers)]
            self._opened: List[int] = []
            if self.world == 1:
                for b in range(self.n_buffers):
                    self.recv[b][0] = self._own[b]
            else:
                mine = torch.tensor(list(handles), dtype=torch.uint8, device=self.device)
                gathered = [torch.empty_like(mine) for _ in range(self.world)]
                dist.all_gather(gathered, mine, group=group)
                for r, t in enumerate(gathered):
                    raw = bytes(t.cpu().tolist())
                    for b in range(self.n_buffers):
                        if r == self.rank:
                            self.recv[b][r] = self._own[b]
                            continue
                        h = _lib.PeerHandle()
                        ctypes.memmove(h.bytes, raw[b * 64:(b + 1) * 64], 64)
                        ptr = ctypes.c_void_p()
                        _lib.call("tgs_peer_buffer_open", ctypes.byref(h), ctypes.byref(ptr))
                        self.recv[b][r] = int(ptr.value)
                        self._opened.append(int(ptr.value))
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._closed = False
        del lib

    def push(self, plan: ExchangePlan, grads: Mapping[str, torch.Tensor], block_row_start,
             parity: int, err: Optional[torch.Tensor] = None) -> int:
        """Stores this rank's tiles into the owners' buffers `parity`.
        Returns the number of rows pushed."""
        B = self.block_size
        n = int(plan.send_blocks.size)
        if n == 0:
            return 0
        starts = _send_starts(plan, block_row_start)
        dst_rank = owner_of(plan.send_blocks, plan.world)
        table = np.concatenate([starts, np.full(n, B, np.int64),
                                plan.send_dst_tiles.astype(np.int64) * B])
        dev = _ops.i64_to_device(table, self.device)
        rank32 = _ops.upload_into(torch.empty(n, dtype=torch.int32, device=self.device),
                                  dst_rank.astype(np.int32))
        args = _lib.GradPushArgs()
        for c, ptr in enumerate(_ops._comp_ptrs(grads, "PeerGradExchange.push")):
            args.comp[c] = ptr
        args.src_start = dev[:n].data_ptr()
        args.row_count = dev[n:2 * n].data_ptr()
        args.dst_row = dev[2 * n:3 * n].data_ptr()
        args.dst_rank = rank32.data_ptr()
        args.n_tiles = n
        args.max_rows = B
        for r in range(plan.world):
            args.recv[r] = self.recv[parity % self.n_buffers][r]
            args.recv_rows[r] = self.capacity_rows
        args.n_ranks = plan.world
        args.err = _lib.ptr(err)
        stream = torch.cuda.current_stream(self.device)
        _lib.call("tgs_grad_push", args, stream.cuda_stream)
        dev.record_stream(stream)
        rank32.record_stream(stream)
        return n * B

    def barrier(self) -> None:
        """Orders every rank's push before the sums that follow on the stream."""
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(self._flag, group=self.group)

    def reduce(self, plan: ExchangePlan, parity: int,
               out: Optional[Mapping[str, torch.Tensor]] = None,
               err: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        """Compact SoA gradients of the owner's visible blocks from buffer
        `parity` (plan.out_blocks order, block_size rows each)."""
        if int(sum(plan.recv_counts)) * self.block_size > self.capacity_rows:
            raise RuntimeError("PeerGradExchange: plan exceeds the receive capacity")
        return _sum_tiles(plan, self._own[parity % self.n_buffers], self.device, out, err)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective: every
        rank calls it, with no push or sum in flight)."""
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                _lib.call("tgs_peer_buffer_close", ptr)
            if self.world > 1:
                import torch.distributed as dist

                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)
            for ptr in self._own:
                _lib.call("tgs_peer_buffer_free", ptr)
        self._opened, self._own = [], []


def _map_peer_components(comps: Mapping[str, torch.Tensor], device: torch.device, group,
                         world: int, rank: int, who: str):
    """Exports this rank's six [rows, width] component tensors (tgs_peer_export:
    IPC handle of the containing allocation + the tensor's offset in it) and
    maps every other rank's (collective over `group`). Returns the [world, 6]
    table of component pointers valid in this process, each rank's row count
    and the opened allocations {handle: base} (closed by the caller)."""
    import ctypes

    import torch.distributed as dist

    own_ptrs = _ops._comp_ptrs(comps, who)
    rows = min(int(comps[n].shape[0]) for n in _ops.COMPONENTS)
    for n, w in _ops.WIDTHS.items():
        t = comps[n]
        if t.device != device or t.numel() != int(t.shape[0]) * w:
            raise RuntimeError(f"{who}: component {n} must be [rows, {w}] on {device}")
    n_comp = len(_ops.COMPONENTS)
    table = np.zeros((world, n_comp), np.int64)
    rows_of = np.zeros(world, np.int64)
    opened: Dict[bytes, int] = {}
    if world == 1:
        table[0] = own_ptrs
        rows_of[0] = rows
        return table, rows_of, opened
    rec = bytearray()
    with torch.cuda.device(device):
        for ptr in own_ptrs:
            h = _lib.PeerHandle()
            off = ctypes.c_int64()
            _lib.call("tgs_peer_export", ptr, ctypes.byref(h), ctypes.byref(off))
            rec += bytes(h.bytes) + int(off.value).to_bytes(8, "little", signed=True)
        rec += rows.to_bytes(8, "little", signed=True)
        mine = torch.tensor(list(rec), dtype=torch.uint8, device=device)
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine, group=group)
        step = 64 + 8
        for r, t in enumerate(gathered):
            raw = bytes(t.cpu().tolist())
            rows_of[r] = int.from_bytes(raw[n_comp * step:n_comp * step + 8], "little",
                                        signed=True)
            if r == rank:
                table[r] = own_ptrs
                continue
            for c in range(n_comp):
                key = raw[c * step:c * step + 64]
                off = int.from_bytes(raw[c * step + 64:(c + 1) * step], "little", signed=True)
                if key not in opened:
                    h = _lib.PeerHandle()
                    ctypes.memmove(h.bytes, key, 64)
                    base = ctypes.c_void_p()
                    _lib.call("tgs_peer_buffer_open", ctypes.byref(h), ctypes.byref(base))
                    opened[key] = int(base.value)
                table[r, c] = opened[key] + off
    return table, rows_of, opened


def _close_peer_mappings(opened: Dict[bytes, int], device: torch.device, group,
                         collective: bool) -> None:
    """Unmaps what _map_peer_components opened (collective: every rank calls
    it with nothing in flight that reads a peer)."""
    torch.cuda.synchronize(device)
    if collective:
        import torch.distributed as dist

        dist.barrier(group=group)
    with torch.cuda.device(device):
        for base in opened.values():
            _lib.call("tgs_peer_buffer_close", base)
    if collective:
        import torch.distributed as dist

        dist.barrier(group=group)


class PeerGradPull:
    """Owner-side gradient reduction fused into the resident Adam update.

    Each rank exports its six gradient component tensors once
    (tgs_peer_export: IPC handle of the containing allocation + offset) and
    maps every other rank's. A step then moves no data of its own: the
    owner's update kernel (tgs_resident_adam_apply_sum, reached through
    GPUResidentAdam.step_pulled) reads each row's contributions from the
    senders' buffers over NVLink and sums them in rank order, so the result
    equals the push / all-to-all path bit for bit. Per step, on the current
    stream of every rank:

        barrier   every rank's gradients of this step are written
        update    count + fused update kernels on each owner
        barrier   no owner still reads; senders may overwrite their gradients

    The gradient tensors stay fixed for the object's life. Rank r's rows hold
    its rendered blocks in ascending block id, block_size rows each (the
    order ExchangePlan.recv_src_tiles refers to).
    """

    def __init__(self, grads: Mapping[str, torch.Tensor], block_size: int, device, group=None):
        import torch.distributed as dist

        self.device = _lib.require_cuda(device, "PeerGradPull")
        self.block_size = int(block_size)
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if self.world > _lib.MAX_PEERS:
            raise RuntimeError(f"PeerGradPull supports at most {_lib.MAX_PEERS} ranks")
        table, self.rows, self._opened = _map_peer_components(
            grads, self.device, group, self.world, self.rank, "PeerGradPull")
        self._finish(table, {"own": dict(grads)}, collective=self.world > 1)

    @classmethod
    def in_process(cls, grads_by_rank: Sequence[Mapping[str, torch.Tensor]], rank: int,
                   block_size: int, device) -> "PeerGradPull":
        """Every rank's gradients live in this process (ranks emulated on one
        GPU, or one process driving several GPUs): no IPC mappings and no
        barriers; gradients on other devices are read through peer access."""
        self = cls.__new__(cls)
        self.device = _lib.require_cuda(device, "PeerGradPull")
        with torch.cuda.device(self.device):
            for g in grads_by_rank:
                other = g["xyz"].device
                if other != self.device:
                    _lib.call("tgs_peer_access_enable", int(other.index))
        self.block_size = int(block_size)
        self.group = None
        self.world = len(grads_by_rank)
        self.rank = int(rank)
        self._opened = {}
        table = np.asarray([_ops._comp_ptrs(g, "PeerGradPull") for g in grads_by_rank], np.int64)
        self.rows = np.asarray([min(int(g[n].shape[0]) for n in _ops.COMPONENTS)
                                for g in grads_by_rank], np.int64)
        self._finish(table, {r: dict(g) for r, g in enumerate(grads_by_rank)}, collective=False)
        return self

    def _finish(self, table: np.ndarray, keep, collective: bool) -> None:
        self._src_dev = _ops.i64_to_device(table.reshape(-1), self.device)
        self._rows_dev = _ops.i64_to_device(self.rows, self.device)
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._grads = keep  # keeps the exported tensors alive
        # cap on the streamed update's CTAs (0 = one per SM): leaves SMs to
        # work on another stream while NVLink bounds the update
        self.max_ctas = 0
        self._collective = collective
        self._closed = False

    def barrier(self) -> None:
        if self._collective:
            import torch.distributed as dist

            dist.all_reduce(self._flag, group=self.group)

    def tables(self, plan: ExchangePlan):
        """Device tables of the fused kernel for `plan` (this rank as owner)."""
        if plan.world != self.world or plan.rank != self.rank:
            raise ValueError("PeerGradPull: plan is for another world/rank")
        B = plan.block_size
        S = plan.n_out
        sender = np.repeat(np.arange(plan.world, dtype=np.int64), plan.recv_counts)
        c_rank = sender[plan.contrib_blocks]
        c_row = plan.recv_src_tiles[plan.contrib_blocks] * B
        if c_row.size and np.any(c_row + B > self.rows[c_rank]):
            raise RuntimeError("PeerGradPull: a contribution lies outside its sender's gradients")
        i64 = _ops.i64_to_device(np.concatenate([np.arange(S + 1, dtype=np.int64) * B,
                                                 plan.contrib_offsets, c_row]), self.device)
        i32 = _ops.upload_into(torch.empty(max(1, c_rank.size), dtype=torch.int32,
                                           device=self.device),
                               c_rank.astype(np.int32) if c_rank.size else np.zeros(1, np.int32))
        return i64, i32

    def apply(self, adam_args, plan: ExchangePlan, stream: int) -> None:
        """acquire barrier -> tgs_resident_adam_apply_sum -> release barrier.
        adam_args: a filled _lib.ResidentAdamArgs (its grad pointers unused)."""
        self.barrier()
        self.launch(adam_args, plan, stream)
        self.barrier()

    def launch(self, adam_args, plan: ExchangePlan, stream: int, tables=None,
               max_ctas: Optional[int] = None) -> None:
        """The fused update alone; the caller provides both barriers.
        tables: the result of tables(plan), when the caller built it earlier.
        max_ctas: cap on the streamed kernel's CTAs (0 = one per SM; None =
        self.max_ctas), to leave SMs to work on another stream."""
        S = plan.n_out
        if int(adam_args.n_rows) != S * plan.block_size:
            raise ValueError("PeerGradPull: rows to update do not match the plan's blocks")
        i64, i32 = tables if tables is not None else self.tables(plan)
        args = _lib.ResidentAdamSumArgs()
        args.adam = adam_args
        args.grad_src = self._src_dev.data_ptr()
        args.grad_rows = self._rows_dev.data_ptr()
        args.n_ranks = self.world
        args.seg_begin = i64[:S + 1].data_ptr()
        args.n_segments = S
        args.contrib_offsets = i64[S + 1:2 * S + 2].data_ptr()
        args.contrib_row = i64[2 * S + 2:].data_ptr()
        args.contrib_rank = i32.data_ptr()
        # start at this rank's share of the rows, so that at any moment the
        # owners pull from different senders
        args.rotate_rows = (self.rank * S // max(1, self.world)) * plan.block_size
        args.max_ctas = int(self.max_ctas if max_ctas is None else max_ctas)
        args.err = adam_args.err
        _lib.call("tgs_resident_adam_apply_sum", args, stream)
        cur = torch.cuda.current_stream(self.device)
        i64.record_stream(cur)
        i32.record_stream(cur)

    def close(self) -> None:
        """Unmaps the peers' gradient buffers (collective: every rank calls it
        with no update in flight)."""
        if self._closed:
            return
        self._closed = True
        _close_peer_mappings(self._opened, self.device, self.group, self._collective)
        self._opened = {}
        self._grads = {}


@dataclass
class GatherPlan:
    """Where a renderer finds the current parameters of the blocks it renders
    next. Blocks this rank owns are read in place from its own arena; every
    other one is copied whole from its owner's arena slot into the render
    rows: remote_blocks[i] lands in rows [i * block_size, (i + 1) *
    block_size) of every component."""
    world: int
    rank: int
    block_size: int
    own_blocks: np.ndarray       # rendered blocks this rank owns, ascending id
    own_slots: np.ndarray        # their slots in this rank's arena
    remote_blocks: np.ndarray    # rendered blocks of other owners, ascending id
    src_slot: np.ndarray         # [len(remote_blocks)] slot in the owner's arena
    owner: np.ndarray            # [len(remote_blocks)] owner rank
    missing: np.ndarray          # rendered blocks resident on no owner (host tier)

    def owner_order(self) -> List[int]:
        """Owners in the order this rank reads them: rank + 1, rank + 2, ...,
        so that at any moment the owners serve different readers."""
        return [(self.rank + d) % self.world for d in range(1, self.world)]


def make_gather_plan(blocks, arena_blocks_by_rank: Sequence[np.ndarray], world: int, rank: int,
                     block_size: int) -> GatherPlan:
    """GatherPlan of this rank for `blocks` (the block ids it renders next).

    arena_blocks_by_rank[o][s] is the block in owner o's arena slot s (-1 for
    a free slot). A block must sit in its owner's arena (owner = id mod
    world) to be gathered; the ones that do not are listed in `missing` and
    come from the host tier instead."""
    blocks = np.unique(np.asarray(blocks, np.int64))
    if len(arena_blocks_by_rank) != world:
        raise ValueError("make_gather_plan: one arena table per rank is needed")
    owner = owner_of(blocks, world)
    slot = np.full(blocks.size, -1, np.int64)
    for o in range(world):
        arena = np.asarray(arena_blocks_by_rank[o], np.int64)
        sel = np.flatnonzero(owner == o)
        if sel.size == 0:
            continue
        held = np.flatnonzero(arena >= 0)
        if held.size and np.any(owner_of(arena[held], world) != o):
            raise ValueError(f"make_gather_plan: rank {o}'s arena holds a block it does not own")
        order = np.argsort(arena[held], kind="stable")
        keys = arena[held][order]
        if keys.size and np.any(keys[1:] == keys[:-1]):
            raise ValueError(f"make_gather_plan: rank {o}'s arena holds a block twice")
        at = np.searchsorted(keys, blocks[sel])
        hit = at < keys.size
        hit[hit] = keys[at[hit]] == blocks[sel][hit]
        slot[sel[hit]] = held[order[at[hit]]]
    found = slot >= 0
    mine = owner == rank
    return GatherPlan(world=world, rank=rank, block_size=int(block_size),
                      own_blocks=blocks[mine & found], own_slots=slot[mine & found],
                      remote_blocks=blocks[~mine & found], src_slot=slot[~mine & found],
                      owner=owner[~mine & found], missing=blocks[~found])


class PeerParamGather:
    """Updated parameters of resident blocks, copied from their owners'
    arenas to the ranks that render them next: the all-gather of changed
    blocks that ownership sharding needs (TideGS trains on one GPU and has
    none). Each rank exports its six arena component tensors once and maps
    every other rank's. A gather, on the current stream of every rank:

        barrier   every owner's update of the blocks is complete
        copies    one tgs_copy_blocks launch per owner (GatherPlan.owner_order):
                  whole block segments, read from the owner's arena over
                  NVLink with bulk copies (no multicast) and stored into this
                  rank's render rows
        barrier   no rank still reads; owners may update their blocks again

    The arena tensors stay fixed for the object's life."""

    def __init__(self, arena: Mapping[str, torch.Tensor], block_size: int, device, group=None):
        import torch.distributed as dist

        self.device = _lib.require_cuda(device, "PeerParamGather")
        self.block_size = int(block_size)
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        table, self.rows, self._opened = _map_peer_components(
            arena, self.device, group, self.world, self.rank, "PeerParamGather")
        self._finish(table, {"own": dict(arena)}, collective=self.world > 1)

    @classmethod
    def in_process(cls, arenas_by_rank: Sequence[Mapping[str, torch.Tensor]], rank: int,
                   block_size: int, device) -> "PeerParamGather":
        """Every rank's arena lives in this process (ranks emulated on one
        GPU, or one process driving several GPUs): no IPC mappings and no
        barriers; arenas on other devices are read through peer access."""
        self = cls.__new__(cls)
        self.device = _lib.require_cuda(device, "PeerParamGather")
        with torch.cuda.device(self.device):
            for a in arenas_by_rank:
                other = a["xyz"].device
                if other != self.device:
                    _lib.call("tgs_peer_access_enable", int(other.index))
        self.block_size = int(block_size)
        self.group = None
        self.world = len(arenas_by_rank)
        self.rank = int(rank)
        self._opened = {}
        table = np.asarray([_ops._comp_ptrs(a, "PeerParamGather") for a in arenas_by_rank],
                           np.int64)
        self.rows = np.asarray([min(int(a[n].shape[0]) for n in _ops.COMPONENTS)
                                for a in arenas_by_rank], np.int64)
        self._finish(table, {r: dict(a) for r, a in enumerate(arenas_by_rank)}, collective=False)
        return self

    def _finish(self, table: np.ndarray, keep, collective: bool) -> None:
        self._table = table
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._arenas = keep  # keeps the exported tensors alive
        self._collective = collective
        self._closed = False

    def barrier(self) -> None:
        if self._collective:
            import torch.distributed as dist

            dist.all_reduce(self._flag, group=self.group)

    def tables(self, plan: GatherPlan) -> List[tuple]:
        """Per owner, in plan.owner_order(): (owner, [3, n] device table of
        source rows, render rows and row counts, n)."""
        if plan.world != self.world or plan.rank != self.rank:
            raise ValueError("PeerParamGather: plan is for another world/rank")
        if plan.block_size != self.block_size:
            raise ValueError("PeerParamGather: plan is for another block size")
        B = self.block_size
        out = []
        dst_index = np.arange(plan.remote_blocks.size, dtype=np.int64)
        for o in plan.owner_order():
            sel = plan.owner == o
            n = int(np.count_nonzero(sel))
            if n == 0:
                continue
            src = plan.src_slot[sel] * B
            if np.any(src + B > self.rows[o]):
                raise RuntimeError(f"PeerParamGather: a slot lies outside rank {o}'s arena")
            t = _ops.i64_to_device(np.stack([src, dst_index[sel] * B, np.full(n, B, np.int64)]),
                                   self.device).view(3, n)
            out.append((o, t, n))
        return out

    def launch(self, dst: Mapping[str, torch.Tensor], plan: GatherPlan, tables=None,
               err: Optional[torch.Tensor] = None) -> int:
        """The copies alone (the caller provides both barriers). dst: six
        render components with at least len(plan.remote_blocks) * block_size
        rows. Returns the rows copied."""
        B = self.block_size
        need = plan.remote_blocks.size * B
        dst_ptrs = _ops._comp_ptrs(dst, "PeerParamGather(dst)")
        for n, w in _ops.WIDTHS.items():
            t = dst[n]
            if t.device != self.device or t.numel() != int(t.shape[0]) * w:
                raise RuntimeError(f"PeerParamGather: render rows {n} must be [rows, {w}] "
                                   f"on {self.device}")
            if int(t.shape[0]) < need:
                raise RuntimeError(f"PeerParamGather: render rows {n} hold {int(t.shape[0])} "
                                   f"rows, the plan needs {need}")
        tables = tables if tables is not None else self.tables(plan)
        stream = torch.cuda.current_stream(self.device)
        copied = 0
        for o, t, n in tables:
            args = _lib.CopyBlocksArgs()
            for c in range(len(_ops.COMPONENTS)):
                args.src_comp[c] = int(self._table[o, c])
                args.dst_comp[c] = dst_ptrs[c]
            args.src_global_ids = None
            args.dst_global_ids = None
            args.src_start = t[0].data_ptr()
            args.dst_start = t[1].data_ptr()
            args.row_count = t[2].data_ptr()
            args.n_blocks = n
            args.max_rows = B
            args.err = _lib.ptr(err)
            _lib.call("tgs_copy_blocks", args, stream.cuda_stream)
            t.record_stream(stream)
            copied += n * B
        return copied

    def gather(self, dst: Mapping[str, torch.Tensor], plan: GatherPlan, tables=None,
               err: Optional[torch.Tensor] = None) -> int:
        """acquire barrier -> copies from every owner -> release barrier."""
        self.barrier()
        copied = self.launch(dst, plan, tables, err)
        self.barrier()
        return copied

    def close(self) -> None:
        """Unmaps the peers' arenas (collective: every rank calls it with no
        gather in flight)."""
        if self._closed:
            return
        self._closed = True
        _close_peer_mappings(self._opened, self.device, self.group, self._collective)
        self._opened = {}
        self._arenas = {}


def exchange_arena_tables(arena_blocks, device, group=None) -> List[np.ndarray]:
    """Every rank's arena table (the block held in each arena slot, -1 for a
    free slot), all-gathered: the input of make_gather_plan. Collective;
    `device` is where the backend wants its tensors (CPU for gloo)."""
    import torch.distributed as dist

    mine = np.asarray(arena_blocks, np.int64).reshape(-1)
    world = dist.get_world_size(group)
    n = torch.tensor([mine.size], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(x.item()) for x in sizes]
    padded = torch.full((max(sizes),), -1, dtype=torch.int64, device=device)
    padded[:mine.size] = torch.from_numpy(mine).to(device)
    out = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(out, padded, group=group)
    return [t.cpu().numpy()[:m].copy() for t, m in zip(out, sizes)]
