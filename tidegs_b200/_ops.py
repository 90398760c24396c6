"""Thin tensor-level wrappers over the block-movement entry points of
libtidegs_b200.so, shared by the working-set classes. Every function enqueues
on the current CUDA stream of the tensors' device and raises on failure."""
from __future__ import annotations

import collections
import threading
from typing import Dict, Iterable, List, Mapping, Optional, Sequence

import numpy as np
import torch

from . import _lib

# Library component order (reference COMPONENT_SPECS order).
COMPONENTS = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")
WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}


def _stream(device: torch.device) -> int:
    return _lib.stream_handle(device)


class _HostTables:
    """Page-locked host copies of small per-step tables, read on the device by
    tgs_copy_small. A table stays referenced until an event recorded after
    the kernel that reads it has completed (the caching host allocator only
    tracks copies it issued itself)."""

    def __init__(self):
        self._lock = threading.Lock()
        self._inflight = collections.deque()

    def stage(self, arr: np.ndarray) -> torch.Tensor:
        with self._lock:
            while self._inflight and self._inflight[0][1].query():
                self._inflight.popleft()
        return torch.from_numpy(arr).pin_memory()

    def retire(self, host: torch.Tensor, stream: torch.cuda.Stream) -> None:
        ev = torch.cuda.Event()
        ev.record(stream)
        with self._lock:
            self._inflight.append((host, ev))


_TABLES = _HostTables()


def upload_into(dst: torch.Tensor, values) -> torch.Tensor:
    """Writes host `values` (numpy-compatible, dst's dtype) into the contiguous
    device tensor dst with a kernel on the current stream, so the upload is
    ordered with the compute work and never waits behind bulk DMA."""
    arr = np.ascontiguousarray(np.asarray(values).reshape(-1))
    if arr.size == 0:
        return dst
    if arr.nbytes != dst.numel() * dst.element_size() or not dst.is_contiguous():
        raise RuntimeError("upload_into: size or layout mismatch")
    host = _TABLES.stage(arr)
    stream = torch.cuda.current_stream(dst.device)
    _lib.call("tgs_copy_small", dst.data_ptr(), host.data_ptr(), arr.nbytes, stream.cuda_stream)
    _TABLES.retire(host, stream)
    return dst


def i64_to_device(values, device: torch.device) -> torch.Tensor:
    """Host ints -> device int64 (kernel upload from a page-locked copy)."""
    arr = np.ascontiguousarray(np.asarray(values, dtype=np.int64).reshape(-1))
    out = torch.empty(arr.size, dtype=torch.int64, device=device)
    if arr.size:
        upload_into(out, arr)
    return out


def _comp_ptrs(components: Mapping[str, torch.Tensor], who: str) -> List[int]:
    out = []
    for name in COMPONENTS:
        t = components[name]
        if t is None:
            raise RuntimeError(f"{who}: component {name} is missing")
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise RuntimeError(f"{who}: component {name} must be contiguous float32")
        out.append(t.data_ptr())
    return out


def unpack_rows(packed: torch.Tensor, layout_code: int, targets: Mapping[str, torch.Tensor],
                target_offset: int, global_ids: Optional[torch.Tensor] = None,
                block_ids: Optional[torch.Tensor] = None, block_size: int = 0,
                err: Optional[torch.Tensor] = None,
                block_dst: Optional[Sequence[int]] = None) -> None:
    """Unpacks packed [rows, 59] into the SoA targets: contiguously at
    target_offset, or, with block_dst (host ints, one per block of
    block_size rows), block k at target row block_dst[k]."""
    n_rows = int(packed.shape[0])
    if n_rows == 0:
        return
    if packed.dtype != torch.float32 or not packed.is_contiguous() or packed.shape[1] != 59:
        raise RuntimeError("unpack_rows: packed rows must be contiguous float32 [rows, 59]")
    target_rows = min(int(targets[n].shape[0]) for n in COMPONENTS)
    dst_dev = None
    if block_dst is not None:
        dst = np.asarray(block_dst, np.int64)
        if block_size <= 0 or dst.size * block_size < n_rows:
            raise ValueError("unpack_rows: block_dst needs one target row per block")
        if dst.size and (dst.min() < 0 or dst.max() + block_size > target_rows):
            raise ValueError("unpack_rows: a block_dst slot lies outside the targets")
        dst_dev = i64_to_device(dst, packed.device)
    elif target_offset < 0 or target_offset + n_rows > target_rows:
        raise ValueError(f"unpack_rows: rows [{target_offset}, {target_offset + n_rows}) "
                         f"outside {target_rows}-row targets")
    args = _lib.UnpackArgs()
    args.packed = packed.data_ptr()
    args.n_rows = n_rows
    args.layout = int(layout_code)
    for c, p in enumerate(_comp_ptrs(targets, "unpack_rows")):
        args.comp[c] = p
    args.target_offset = int(target_offset)
    args.global_ids = _lib.ptr(global_ids)
    args.block_ids = _lib.ptr(block_ids)
    args.block_size = int(block_size)
    args.err = _lib.ptr(err)
    args.block_dst = _lib.ptr(dst_dev)
    _lib.call("tgs_unpack_rows", args, _stream(packed.device))
    if dst_dev is not None:
        _keepalive(dst_dev, packed.device)


def copy_blocks(src: Mapping[str, torch.Tensor], src_gids: Optional[torch.Tensor],
                dst: Mapping[str, torch.Tensor], dst_gids: Optional[torch.Tensor],
                src_starts: Sequence[int], dst_starts: Sequence[int], row_counts: Sequence[int],
                device: torch.device, err: Optional[torch.Tensor] = None) -> int:
    n = len(row_counts)
    if n == 0:
        return 0
    plan = i64_to_device(np.stack([np.asarray(src_starts, np.int64),
                                   np.asarray(dst_starts, np.int64),
                                   np.asarray(row_counts, np.int64)]), device).view(3, n)
    args = _lib.CopyBlocksArgs()
    for c, p in enumerate(_comp_ptrs(src, "copy_blocks(src)")):
        args.src_comp[c] = p
    for c, p in enumerate(_comp_ptrs(dst, "copy_blocks(dst)")):
        args.dst_comp[c] = p
    copy_ids = src_gids is not None and dst_gids is not None
    args.src_global_ids = src_gids.data_ptr() if copy_ids else None
    args.dst_global_ids = dst_gids.data_ptr() if copy_ids else None
    args.src_start = plan[0].data_ptr()
    args.dst_start = plan[1].data_ptr()
    args.row_count = plan[2].data_ptr()
    args.n_blocks = n
    args.max_rows = int(max(row_counts))
    args.err = _lib.ptr(err)
    _lib.call("tgs_copy_blocks", args, _stream(device))
    _keepalive(plan, device)
    return int(sum(row_counts))


def _keepalive(t: torch.Tensor, device: torch.device) -> None:
    """Marks `t` as used by the current stream, so the caching allocator keeps
    its memory until the kernel enqueued there has read it, whichever stream
    frees it."""
    t.record_stream(torch.cuda.current_stream(device))


def fill_global_ids(dst: torch.Tensor, offset: int, block_ids: torch.Tensor, n_rows: int,
                    block_size: int) -> None:
    if n_rows == 0:
        return
    if offset < 0 or offset + n_rows > dst.numel() or not dst.is_contiguous():
        raise ValueError(f"fill_global_ids: rows [{offset}, {offset + n_rows}) outside a "
                         f"{dst.numel()}-row destination")
    if block_ids.numel() * block_size < n_rows:
        raise ValueError(f"fill_global_ids: {block_ids.numel()} block ids cannot cover "
                         f"{n_rows} rows of {block_size}")
    _lib.call("tgs_fill_global_ids", dst.data_ptr(), int(offset), block_ids.data_ptr(),
              int(n_rows), int(block_size), _stream(dst.device))


def build_block_starts(items: Iterable, num_blocks: int, device: torch.device) -> torch.Tensor:
    """[num_blocks] int64: start of each listed (block_id, start) pair, -1 elsewhere."""
    pairs = [(int(b), int(s)) for b, s in items if 0 <= int(b) < num_blocks]
    out = torch.empty(max(num_blocks, 0), dtype=torch.int64, device=device)
    if num_blocks == 0:
        return out
    if pairs:
        arr = i64_to_device(np.asarray(pairs, np.int64).T.copy(), device).view(2, len(pairs))
        _lib.call("tgs_build_block_starts", out.data_ptr(), int(num_blocks), arr[0].data_ptr(),
                  arr[1].data_ptr(), len(pairs), _stream(device))
        _keepalive(arr, device)
    else:
        _lib.call("tgs_build_block_starts", out.data_ptr(), int(num_blocks), None, None, 0,
                  _stream(device))
    return out


def global_to_local(global_ids: torch.Tensor, block_starts: torch.Tensor,
                    block_size: int) -> torch.Tensor:
    gids = global_ids.to(device=block_starts.device, dtype=torch.int64).contiguous()
    out = torch.empty_like(gids)
    if gids.numel() == 0:
        return out
    _lib.call("tgs_global_to_local", out.data_ptr(), gids.data_ptr(), gids.numel(),
              block_starts.data_ptr(), block_starts.numel(), int(block_size),
              _stream(block_starts.device))
    return out.view(global_ids.shape)


def global_to_local_compact(global_ids: torch.Tensor, block_starts: torch.Tensor,
                            block_size: int) -> torch.Tensor:
    """global_to_local keeping only resident ids, in input order (one sync
    to read the count, as boolean-mask indexing also does)."""
    device = block_starts.device
    gids = global_ids.to(device=device, dtype=torch.int64).contiguous().view(-1)
    n = gids.numel()
    if n == 0:
        return torch.empty(0, dtype=torch.int64, device=device)
    lib = _lib.load()
    words = int(lib.tgs_compact_scratch_words(n))
    scratch = torch.empty(words + 1, dtype=torch.int64, device=device)
    out = torch.empty(n, dtype=torch.int64, device=device)
    _lib.call("tgs_global_to_local_compact", out.data_ptr(), scratch[words:].data_ptr(),
              gids.data_ptr(), n, block_starts.data_ptr(), block_starts.numel(),
              int(block_size), scratch.data_ptr(), _stream(device))
    count = int(scratch[words].item())
    return out[:count]


def pack_rows(sources: Mapping[str, torch.Tensor], src_starts: Sequence[int],
              row_counts: Sequence[int], out: torch.Tensor, layout_code: int,
              err: Optional[torch.Tensor] = None) -> List[torch.Tensor]:
    """Packs plan k's rows [src_starts[k], +row_counts[k]) into consecutive
    rows of `out` ([sum rows, 59]). Returns device tensors to keep alive."""
    n = len(row_counts)
    if n == 0:
        return []
    device = out.device
    out_starts = np.zeros(n, np.int64)
    if n > 1:
        out_starts[1:] = np.cumsum(np.asarray(row_counts[:-1], np.int64))
    plan = i64_to_device(np.stack([np.asarray(src_starts, np.int64),
                                   np.asarray(row_counts, np.int64), out_starts]),
                         device).view(3, n)
    args = _lib.PackArgs()
    for c, p in enumerate(_comp_ptrs(sources, "pack_rows")):
        args.comp[c] = p
    args.src_start = plan[0].data_ptr()
    args.row_count = plan[1].data_ptr()
    args.out_start = plan[2].data_ptr()
    args.n_plans = n
    args.max_rows = int(max(row_counts))
    args.out = out.data_ptr()
    args.layout = int(layout_code)
    args.err = _lib.ptr(err)
    _lib.call("tgs_pack_rows", args, _stream(device))
    return [plan]


def block_bounds(xyz: torch.Tensor, starts: Sequence[int], counts: Sequence[int],
                 out: torch.Tensor) -> List[torch.Tensor]:
    n = len(counts)
    if n == 0:
        return []
    device = xyz.device
    plan = i64_to_device(np.stack([np.asarray(starts, np.int64),
                                   np.asarray(counts, np.int64)]), device).view(2, n)
    if not xyz.is_contiguous() or xyz.dtype != torch.float32:
        raise RuntimeError("block_bounds: xyz must be contiguous float32")
    _lib.call("tgs_block_bounds", xyz.data_ptr(), plan[0].data_ptr(), plan[1].data_ptr(), n,
              out.data_ptr(), _stream(device))
    return [plan]


# ---------------------------------------------------------------------------
# Dirty bitmap
# ---------------------------------------------------------------------------
def bitmap_words(num_blocks: int) -> int:
    return (max(num_blocks, 0) + 31) // 32


def dirty_mark(bitmap: torch.Tensor, ids: Sequence[int], value: bool) -> None:
    """Sets (value) or clears the bits of ids; ids beyond the bitmap are
    ignored."""
    if len(ids) == 0:
        return
    dev_ids = i64_to_device(ids, bitmap.device)
    _lib.call("tgs_dirty_mark", bitmap.data_ptr(), bitmap.numel() * 32, dev_ids.data_ptr(),
              len(ids), 1 if value else 0, _stream(bitmap.device))
    _keepalive(dev_ids, bitmap.device)


class PendingIds:
    """A device-side id list on its way to page-locked host memory: `wait()`
    blocks until the copy has landed and returns the ids."""

    def __init__(self, host: Optional[torch.Tensor], event, keep=()):
        self._host, self._event, self._keep = host, event, keep

    def wait(self) -> List[int]:
        if self._host is None:
            return []
        self._event.synchronize()
        host = self._host.numpy()
        return host[1:1 + int(host[0])].tolist()


def dirty_select_async(bitmap: torch.Tensor, ids: Sequence[int]) -> PendingIds:
    """Enqueues the order-preserving dirty compaction of `ids` and the copy of
    its result to the host on the current stream; the caller keeps enqueuing
    work and collects the ids with `wait()`."""
    if len(ids) == 0:
        return PendingIds(None, None)
    device = bitmap.device
    n = len(ids)
    dev_ids = i64_to_device(ids, device)
    out = torch.empty(n + 1, dtype=torch.int64, device=device)
    _lib.call("tgs_dirty_select", bitmap.data_ptr(), bitmap.numel() * 32, dev_ids.data_ptr(), n,
              out[1:].data_ptr(), out[:1].data_ptr(), _stream(device))
    host = torch.empty(n + 1, dtype=torch.int64, pin_memory=True)
    host.copy_(out, non_blocking=True)
    event = torch.cuda.Event()
    event.record(torch.cuda.current_stream(device))
    return PendingIds(host, event, (dev_ids, out))


def dirty_select(bitmap: torch.Tensor, ids: Sequence[int]) -> List[int]:
    return dirty_select_async(bitmap, ids).wait()


def dirty_list(bitmap: torch.Tensor, num_blocks: int) -> List[int]:
    device = bitmap.device
    out = torch.empty(num_blocks + 1, dtype=torch.int64, device=device)
    _lib.call("tgs_dirty_list", bitmap.data_ptr(), int(num_blocks), out[1:].data_ptr(),
              out[:1].data_ptr(), _stream(device))
    host = out.cpu().numpy()
    return host[1:1 + int(host[0])].tolist()


def h2d_blocks(dst_ptrs: Sequence[int], src_ptrs: Sequence[int], nbytes: Sequence[int],
               device: torch.device) -> None:
    import ctypes as C
    n = len(nbytes)
    if n == 0:
        return
    dst = (C.c_void_p * n)(*dst_ptrs)
    src = (C.c_void_p * n)(*src_ptrs)
    sizes = (C.c_int64 * n)(*nbytes)
    _lib.call("tgs_h2d_blocks", dst, src, sizes, n, _stream(device))


def d2h_blocks(dst_ptrs: Sequence[int], src_ptrs: Sequence[int], nbytes: Sequence[int],
               device: torch.device) -> None:
    """One device-to-host DMA per block on the current stream."""
    import ctypes as C
    n = len(nbytes)
    if n == 0:
        return
    dst = (C.c_void_p * n)(*dst_ptrs)
    src = (C.c_void_p * n)(*src_ptrs)
    sizes = (C.c_int64 * n)(*nbytes)
    _lib.call("tgs_d2h_blocks", dst, src, sizes, n, _stream(device))
