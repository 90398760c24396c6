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
                code runs on gloo for CPU tests);
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

    @property
    def n_out(self) -> int:
        return int(self.out_blocks.size)


def make_plan(visible_by_rank: Sequence[Sequence[int]], world: int, rank: int, block_size: int,
              out_order: Optional[Mapping[int, int]] = None) -> ExchangePlan:
    """Builds this rank's send/receive plan.

    visible_by_rank[r] = blocks whose gradients rank r produced this step.
    out_order (optional) maps each owned block to its sort key in the owner's
    gradient rows (for example the start row of its resident slice, so that
    the owner's local row ids come out ascending); default: block id.
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
    recv_lists = [v[owner_of(v, world) == rank] for v in vis]
    recv_counts = [int(x.size) for x in recv_lists]
    recv_blocks = (np.concatenate(recv_lists) if recv_lists else np.zeros(0, np.int64))
    # group received tiles by block; a stable sort keeps sender order inside a block
    idx = np.argsort(recv_blocks, kind="stable")
    sorted_ids = recv_blocks[idx]
    uniq, first = np.unique(sorted_ids, return_index=True)
    counts = np.diff(np.append(first, sorted_ids.size))
    if out_order is not None:
        missing = [int(b) for b in uniq if int(b) not in out_order]
        if missing:
            raise KeyError(f"blocks {missing[:8]} have no position in the owner's rows")
        keys = np.asarray([out_order[int(b)] for b in uniq], dtype=np.int64)
        perm = np.argsort(keys, kind="stable")
    else:
        perm = np.arange(uniq.size)
    out_blocks = uniq[perm]
    offsets = np.zeros(uniq.size + 1, np.int64)
    pieces = []
    for k, u in enumerate(perm):
        pieces.append(idx[first[u]:first[u] + counts[u]])
        offsets[k + 1] = offsets[k] + counts[u]
    contrib = np.concatenate(pieces) if pieces else np.zeros(0, np.int64)
    return ExchangePlan(world, rank, int(block_size), send_blocks, send_counts, recv_blocks,
                        recv_counts, out_blocks, offsets, contrib.astype(np.int64))


class BlockGradExchange:
    """Runs a plan: pack -> all-to-all -> ordered sum on the owner."""

    def __init__(self, block_size: int, group=None, device: Optional[torch.device] = None):
        self.block_size = int(block_size)
        self.group = group
        self.device = device

    def pack(self, plan: ExchangePlan, grads: Mapping[str, torch.Tensor],
             block_row_start: Mapping[int, int], out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Gathers the rows of each sent block (block_row_start[b] = first
        row of block b in the compact gradient tensors) into UNIFIED tiles."""
        n = int(plan.send_blocks.size) * self.block_size
        dev = grads["xyz"].device
        if out is None:
            out = torch.empty((n, 59), dtype=torch.float32, device=dev)
        if n:
            starts = [int(block_row_start[int(b)]) for b in plan.send_blocks]
            refs = _ops.pack_rows(grads, starts, [self.block_size] * len(starts), out[:n],
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
        B = self.block_size
        dev = recv.device
        rows = plan.n_out * B
        if out is None:
            out = {n: torch.empty((rows, w), dtype=torch.float32, device=dev)
                   for n, w in _ops.WIDTHS.items()}
        else:
            out = {n: t[:rows] for n, t in out.items()}
        if plan.n_out == 0:
            return out
        tables = _ops.i64_to_device(np.concatenate([plan.contrib_offsets, plan.contrib_blocks]),
                                    dev)
        args = _lib.BlockSumArgs()
        args.recv = recv.data_ptr()
        args.n_recv_blocks = int(sum(plan.recv_counts))
        args.contrib_offsets = tables.data_ptr()
        args.contrib_blocks = tables[plan.n_out + 1:].data_ptr()
        args.n_out = plan.n_out
        args.block_size = B
        for c, name in enumerate(_ops.COMPONENTS):
            args.out[c] = out[name].data_ptr()
        args.err = _lib.ptr(err)
        _lib.call("tgs_block_grad_sum", args, _lib.stream_handle(dev))
        tables.record_stream(torch.cuda.current_stream(dev))
        return out
