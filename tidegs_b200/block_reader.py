"""Block reader boundary: the source side of resident-slot materialization.

Mirrors storage/block_reader.py of TideGS (BlockLayout :35-44, BlockBatch
:47-52, _pack_block_batch :55-87, BlockReader protocol :90-119,
UnifiedParamsBlockReader :122-176, parse_block_row_components :239-270) so
the materialization path accepts the same readers. Readers from the
reference package work unchanged: layouts are compared by their string value
("unified" / "cache"), not by enum identity.

Added here: `PinnedBlockPool`, a page-locked host pool whose blocks the
materialization path copies to the device with one DMA per block, skipping
the CPU-side concatenation of `read_batch` (block_reader.py:55-87).
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import Dict, List, Optional, Protocol, Sequence, runtime_checkable

import numpy as np
import torch

from . import _lib


class BlockLayout(Enum):
    """Column order of a 59-wide block tensor."""

    UNIFIED = "unified"  # xyz | opacity | scaling | rotation | dc | rest
    CACHE = "cache"      # xyz | scaling  | rotation | opacity  | dc | rest


def layout_code(layout) -> int:
    """Library layout code for a BlockLayout of either package (or a string)."""
    value = getattr(layout, "value", layout)
    if value == "unified":
        return _lib.LAYOUT_UNIFIED
    if value == "cache":
        return _lib.LAYOUT_CACHE
    raise ValueError(f"Unsupported block layout: {layout!r}")


@dataclass(frozen=True)
class BlockBatch:
    tensor: torch.Tensor
    block_ids: tuple
    block_slices: Dict[int, slice]
    layout: BlockLayout


def _pack_block_batch(
    blocks: Dict[int, torch.Tensor],
    block_ids: Sequence[int],
    layout,
    out: Optional[torch.Tensor] = None,
) -> BlockBatch:
    ordered_ids = tuple(int(block_id) for block_id in block_ids)
    missing = [block_id for block_id in ordered_ids if block_id not in blocks]
    if missing:
        raise KeyError(f"BlockReader omitted blocks; first missing={missing[:8]}")
    pieces = [blocks[block_id] for block_id in ordered_ids]
    total_rows = sum(int(piece.shape[0]) for piece in pieces)
    if out is None:
        out = torch.empty((total_rows, 59), dtype=torch.float32)
    elif out.device.type != "cpu" or out.dim() != 2 or tuple(out.shape) != (total_rows, 59):
        raise ValueError(
            f"BlockBatch output must be CPU ({total_rows}, 59); got {tuple(out.shape)} "
            f"on {out.device}"
        )
    if len(pieces) == 1:
        out.copy_(pieces[0])
    elif pieces:
        torch.cat(pieces, dim=0, out=out)
    block_slices = {}
    offset = 0
    for block_id, piece in zip(ordered_ids, pieces):
        nxt = offset + int(piece.shape[0])
        block_slices[block_id] = slice(offset, nxt)
        offset = nxt
    return BlockBatch(out, ordered_ids, block_slices, layout)


@runtime_checkable
class BlockReader(Protocol):
    total_gaussians: int
    block_size: int
    num_blocks: int
    layout: BlockLayout

    def read_blocks(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        ...

    def read_batch(self, block_ids: List[int], out: Optional[torch.Tensor] = None) -> BlockBatch:
        ...

    def hint_future(self, block_ids: List[int]) -> int:
        ...

    def contains_block(self, block_id: int) -> bool:
        ...


class UnifiedParamsBlockReader:
    """Serves blocks as zero-copy views of a CPU (N, 59) UNIFIED table."""

    layout = BlockLayout.UNIFIED

    def __init__(self, unified_params: torch.Tensor, block_size: int):
        if unified_params is None:
            raise ValueError("UnifiedParamsBlockReader requires a non-None unified_params tensor")
        if unified_params.dim() != 2 or unified_params.shape[1] != 59:
            raise ValueError(
                f"UnifiedParamsBlockReader expects (N, 59) tensor; got shape {tuple(unified_params.shape)}"
            )
        if unified_params.device.type != "cpu":
            raise ValueError(
                f"UnifiedParamsBlockReader expects a CPU tensor; got device={unified_params.device}"
            )
        self._unified_params = unified_params
        self.block_size = int(block_size)
        self.total_gaussians = int(unified_params.shape[0])
        self.num_blocks = (self.total_gaussians + self.block_size - 1) // self.block_size

    def read_blocks(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        out: Dict[int, torch.Tensor] = {}
        data = self._unified_params.data
        for bid in block_ids:
            bid = int(bid)
            if bid < 0 or bid >= self.num_blocks:
                continue
            start = bid * self.block_size
            end = min(start + self.block_size, self.total_gaussians)
            if end > start:
                out[bid] = data[start:end]
        return out

    def read_batch(self, block_ids: List[int], out: Optional[torch.Tensor] = None) -> BlockBatch:
        return _pack_block_batch(self.read_blocks(block_ids), block_ids, self.layout, out)

    def hint_future(self, block_ids: List[int]) -> int:
        return 0

    def contains_block(self, block_id: int) -> bool:
        return 0 <= int(block_id) < self.num_blocks


class PinnedBlockPool:
    """Page-locked host pool of `pool_blocks` packed blocks in one layout.

    Scene block `b` is stored in pool entry `b % pool_blocks` (the pool may be
    smaller than the scene, as in a host cache that holds a window of it).
    `read_blocks_pinned` hands out page-locked views, which the materializer
    copies to the device block by block; `read_blocks`/`read_batch` keep the
    BlockReader protocol for every other caller.
    """

    def __init__(self, data: torch.Tensor, block_size: int, total_gaussians: int,
                 layout=BlockLayout.CACHE):
        if data.dim() != 3 or data.shape[2] != 59 or data.shape[1] != block_size:
            raise ValueError(f"PinnedBlockPool expects (blocks, {block_size}, 59); got "
                             f"{tuple(data.shape)}")
        if data.device.type != "cpu":
            raise ValueError("PinnedBlockPool data must be a CPU tensor")
        self._data = data if data.is_pinned() else data.pin_memory()
        self.block_size = int(block_size)
        self.total_gaussians = int(total_gaussians)
        self.num_blocks = (self.total_gaussians + self.block_size - 1) // self.block_size
        self.pool_blocks = int(data.shape[0])
        self.layout = layout

    def _rows(self, bid: int) -> int:
        return min(self.block_size, self.total_gaussians - bid * self.block_size)

    def entry(self, block_id: int) -> torch.Tensor:
        return self._data[int(block_id) % self.pool_blocks]

    def block_host_pointers(self, block_ids):
        """(host addresses, row counts) of the listed blocks as int64 numpy
        arrays, computed without creating per-block tensors; invalid ids
        raise KeyError like an omitted block."""
        ids = np.asarray(block_ids, dtype=np.int64)
        bad = ids[(ids < 0) | (ids >= self.num_blocks)]
        rows = np.minimum(self.block_size, self.total_gaussians - ids * self.block_size)
        if bad.size or np.any(rows <= 0):
            raise KeyError(f"BlockReader omitted blocks; first missing={bad[:8].tolist()}")
        entry_bytes = self.block_size * 59 * 4
        ptrs = self._data.data_ptr() + (ids % self.pool_blocks) * entry_bytes
        return ptrs.astype(np.int64), rows.astype(np.int64)

    def read_blocks_pinned(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        out = {}
        for bid in block_ids:
            bid = int(bid)
            if 0 <= bid < self.num_blocks and self._rows(bid) > 0:
                out[bid] = self.entry(bid)[: self._rows(bid)]
        return out

    def read_blocks(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        return self.read_blocks_pinned(block_ids)

    def read_batch(self, block_ids: List[int], out: Optional[torch.Tensor] = None) -> BlockBatch:
        valid = [int(b) for b in block_ids if 0 <= int(b) < self.num_blocks]
        return _pack_block_batch(self.read_blocks(valid), valid, self.layout, out)

    def write_block(self, block_id: int, rows: torch.Tensor) -> None:
        self.entry(block_id)[: rows.shape[0]].copy_(rows)

    def hint_future(self, block_ids: List[int]) -> int:
        return 0

    def contains_block(self, block_id: int) -> bool:
        return 0 <= int(block_id) < self.num_blocks


def parse_block_row_components(block_tensor: torch.Tensor, layout) -> Dict[str, torch.Tensor]:
    if block_tensor.dim() != 2 or block_tensor.shape[1] != 59:
        raise ValueError(
            f"parse_block_row_components expects (rows, 59) tensor; got shape {tuple(block_tensor.shape)}"
        )
    cols = component_columns(layout)
    return {name: block_tensor[:, sl] for name, sl in cols.items()}


def component_columns(layout) -> Dict[str, slice]:
    """Column slices of the six components in a packed row of `layout`."""
    if layout_code(layout) == _lib.LAYOUT_UNIFIED:
        return {
            "xyz": slice(0, 3), "opacity": slice(3, 4), "scaling": slice(4, 7),
            "rotation": slice(7, 11), "features_dc": slice(11, 14), "features_rest": slice(14, 59),
        }
    return {
        "xyz": slice(0, 3), "scaling": slice(3, 6), "rotation": slice(6, 10),
        "opacity": slice(10, 11), "features_dc": slice(11, 14), "features_rest": slice(14, 59),
    }


__all__ = [
    "BlockLayout", "BlockBatch", "BlockReader", "UnifiedParamsBlockReader", "PinnedBlockPool",
    "parse_block_row_components", "component_columns", "layout_code",
]
