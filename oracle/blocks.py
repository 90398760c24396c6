"""CPU restatements of the block data movement -- test infrastructure only.

Each function is exact integer / byte work and must match the device bit for
bit. References (strategies/tide_engine/...):
  unpack_rows       double_buffer_gpu.py:150-209 (+ id fill :130-148)
  copy_blocks       double_buffer_gpu.py:40-128, :811-872
  build_block_starts / global_to_local   double_buffer_gpu.py:212-256
  pack_rows         gpu_working_set.py:35-86, plans :913-924
  block_bounds      gpu_working_set.py:88-115, plans :998-1012
  dirty_*           double_buffer_gpu.py:494-543
"""
from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np

WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}
UNIFIED = {"xyz": 0, "opacity": 3, "scaling": 4, "rotation": 7, "features_dc": 11,
           "features_rest": 14}
CACHE = {"xyz": 0, "scaling": 3, "rotation": 6, "opacity": 10, "features_dc": 11,
         "features_rest": 14}


def columns(layout: str) -> Dict[str, int]:
    return UNIFIED if layout == "unified" else CACHE


def unpack_rows(packed: np.ndarray, layout: str, targets: Dict[str, np.ndarray], offset: int,
                gids: np.ndarray = None, block_ids: Sequence[int] = (), block_size: int = 0):
    cols = columns(layout)
    n = packed.shape[0]
    for name, w in WIDTHS.items():
        targets[name][offset:offset + n] = packed[:, cols[name]:cols[name] + w]
    if gids is not None:
        r = np.arange(n, dtype=np.int64)
        pos = r // block_size
        gids[offset:offset + n] = np.asarray(block_ids, np.int64)[pos] * block_size + r % block_size


def copy_blocks(src: Dict[str, np.ndarray], src_gids, dst: Dict[str, np.ndarray], dst_gids,
                src_starts, dst_starts, counts):
    for s, d, n in zip(src_starts, dst_starts, counts):
        for name in WIDTHS:
            dst[name][d:d + n] = src[name][s:s + n]
        if src_gids is not None and dst_gids is not None:
            dst_gids[d:d + n] = src_gids[s:s + n]


def build_block_starts(items, num_blocks: int) -> np.ndarray:
    out = np.full(num_blocks, -1, np.int64)
    for b, s in items:
        if 0 <= b < num_blocks:
            out[b] = s
    return out


def global_to_local(gids: np.ndarray, block_starts: np.ndarray, block_size: int) -> np.ndarray:
    gids = np.asarray(gids, np.int64)
    nb = block_starts.shape[0]
    b = np.floor_divide(gids, block_size)
    within = gids - b * block_size
    safe = np.clip(b, 0, nb - 1)
    starts = block_starts[safe]
    out = starts + within
    out[(b != safe) | (starts < 0)] = -1
    return out


def pack_rows(sources: Dict[str, np.ndarray], src_starts, counts, layout: str = "cache"):
    cols = columns(layout)
    total = int(sum(counts))
    out = np.empty((total, 59), np.float32)
    o = 0
    for s, n in zip(src_starts, counts):
        for name, w in WIDTHS.items():
            out[o:o + n, cols[name]:cols[name] + w] = sources[name][s:s + n]
        o += n
    return out


def writeback_plans(block_ids, block_to_slice, block_size: int, num_total: int):
    plans, starts = [], []
    for b in sorted(set(int(x) for x in block_ids)):
        sl = block_to_slice.get(b)
        if sl is None:
            continue
        n = min(min(block_size, num_total - b * block_size), sl.stop - sl.start)
        if n <= 0:
            continue
        plans.append((b, n))
        starts.append(sl.start)
    return plans, starts


def block_bounds(xyz: np.ndarray, starts, counts) -> np.ndarray:
    out = np.empty((len(counts), 6), np.float32)
    for k, (s, n) in enumerate(zip(starts, counts)):
        rows = xyz[s:s + n]
        out[k, :3] = rows.min(axis=0)
        out[k, 3:] = rows.max(axis=0)
    return out


def block_grad_sum(recv: np.ndarray, offsets, contrib, block_size: int) -> Dict[str, np.ndarray]:
    """Owner-side sum of exchanged [block_size, 59] UNIFIED tiles, added in
    listed (sender) order one fp32 addition at a time, returned as SoA
    components (rows of output block k at k*block_size)."""
    n_out = len(offsets) - 1
    acc = np.empty((n_out * block_size, 59), np.float32)
    for k in range(n_out):
        tiles = [recv[j * block_size:(j + 1) * block_size] for j in contrib[offsets[k]:offsets[k + 1]]]
        s = tiles[0].copy()
        for t in tiles[1:]:
            s = (s + t).astype(np.float32)
        acc[k * block_size:(k + 1) * block_size] = s
    return {n: acc[:, UNIFIED[n]:UNIFIED[n] + w].copy() for n, w in WIDTHS.items()}


class DirtyBitmap:
    """Reference semantics of the dirty-block bitmap."""

    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self.bits = np.zeros(num_blocks, bool)

    def _valid(self, ids) -> List[int]:
        return sorted(set(int(b) for b in ids if 0 <= int(b) < self.num_blocks))

    def mark(self, ids) -> int:
        v = self._valid(ids)
        self.bits[v] = True
        return len(v)

    def for_eviction(self, ids) -> List[int]:
        v = self._valid(ids)
        return [b for b in v if self.bits[b]]

    def dirty(self) -> List[int]:
        return np.nonzero(self.bits)[0].tolist()

    def written_back(self, ids) -> None:
        self.bits[self._valid(ids)] = False
