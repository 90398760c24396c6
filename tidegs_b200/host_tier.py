"""Host tier of the block path: the RAM block cache between the GPU working
set and the on-disk block log, and the block log's data path.

Counterparts in the reference (same constructor arguments, methods, return
values, statistics keys and error conditions):

* `PinnedBlockCache` — storage/tiered_cache_manager.py `TieredCacheManager`:
  lookup and single-flight SSD reads (:181-283), dirty flush and the flush
  worker (:284-374), future prefetch and its worker (:375-422, :734-783),
  upserts (:499-600), dirty submission (:601-636), urgent prefetch
  (:637-732), LRU eviction (:785-860), flush_all / stats / shutdown
  (:861-970).
* `BlockLogStore` — storage/log_storage_manager.py `LogStorageManager`, the
  data path of its raw fp32 block format: base-file index (:169-202),
  grouped reads (:204-291), append-only patches (:293-395), statistics
  (:747-764).
* `CachedBlockReader` — storage/block_reader.py:179-236
  `TieredCacheBlockReader`.

What differs by design:

* Every cached block lives in an entry of ONE page-locked slab
  (`[capacity, block_size, point_dim]` fp32) instead of a tensor per block.
  The device reads an entry with one DMA (`block_host_pointers`) and the
  write-back DMA lands in a fresh entry (`reserve_writeback` /
  `commit_writeback`, used by `GPUWorkingSet.stage_updated_blocks(...,
  host_cache=...)`): no CPU concatenation and no CPU copy of the payload
  (the reference copies every write-back batch into a new slab,
  tiered_cache_manager.py:524-599).
* The block log reads straight into slab entries (`os.preadv`) and writes
  patches straight from them (`os.write` of the entry memory): no
  intermediate `bytes` objects.
* Entries are recycled: an entry returns to the free list when neither the
  cache nor the flushing buffer references it, and is reused only after the
  DMA reads recorded on it (`note_dma_reads`) have completed. Views handed
  out by `prefetch` therefore stay valid until their block has left the
  cache and its entry has been reused.

Out of scope (storage-engine lifecycle, not the data path): patch
compaction, checkpoint manifests, free-space reserves, the legacy
`sync_from_gpu` queue.
"""
from __future__ import annotations

import os
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass
from pathlib import Path
from queue import Empty, Full, Queue
from typing import Dict, Iterable, List, Optional, Sequence, Set, Tuple

import numpy as np
import torch

from .block_reader import BlockLayout, _pack_block_batch

__all__ = ["BlockLocation", "BlockLogStore", "PinnedBlockCache", "CachedBlockReader"]


# ---------------------------------------------------------------------------
# Block log (log_storage_manager.py)
# ---------------------------------------------------------------------------
@dataclass
class BlockLocation:
    """Where the current version of a block lives (log_storage_manager.py:23-29)."""
    file_id: int  # 0 = base file, 1+ = patch files
    offset: int   # byte offset in the file
    size: int     # bytes
    version: int  # 0 for the base file, +1 per patch that rewrote the block


def _byte_view(t: torch.Tensor) -> memoryview:
    """Writable byte view of a contiguous CPU tensor's memory."""
    return memoryview(t.numpy()).cast("B")


class BlockLogStore:
    """Raw fp32 block log: `base_file.bin` holds block b at b * bytes_per_block;
    every `write_patch` appends a new file `patch_<id:06d>_<usec>.bin` with
    the written blocks in ascending id order and points the index at them
    (log_storage_manager.py:31-122, :293-395)."""

    def __init__(self, storage_dir: str, block_size: int, num_blocks: int, point_dim: int = 59,
                 dtype: torch.dtype = torch.float32, verbose: bool = True,
                 max_patch_files: int = 16, max_patch_gb: float = 64.0,
                 min_free_gb: float = 64.0, read_threads: int = 4):
        self.storage_dir = Path(storage_dir)
        self.storage_dir.mkdir(parents=True, exist_ok=True)
        self.block_size = int(block_size)
        self.num_blocks = int(num_blocks)
        self.point_dim = int(point_dim)
        self.dtype = dtype
        self.verbose = bool(verbose)
        self.bytes_per_point = self.point_dim * torch.finfo(dtype).bits // 8
        self.bytes_per_block = self.block_size * self.bytes_per_point
        # compaction / free-space settings are kept for signature parity only
        self.max_patch_files = max(2, int(max_patch_files))
        self.max_stale_patch_bytes = max(0, int(float(max_patch_gb) * (1024 ** 3)))
        self.min_free_bytes = max(0, int(float(min_free_gb) * (1024 ** 3)))
        self.read_threads = max(1, int(read_threads))

        self.index: Dict[int, BlockLocation] = {}
        self.index_lock = threading.Lock()
        self.file_paths: Dict[int, Path] = {0: self.storage_dir / "base_file.bin"}
        self._fds: Dict[int, int] = {}
        self._fd_lock = threading.Lock()
        self.next_patch_id = 1
        self.patch_counter_lock = threading.Lock()
        self._write_lock = threading.RLock()
        self.stats = {
            "reads": 0, "writes": 0, "patches_created": 0, "compactions": 0,
            "compaction_input_bytes": 0, "compaction_output_bytes": 0,
            "compaction_reclaimed_bytes": 0, "compactions_deferred": 0,
        }
        self._initialize_index()

    def _log(self, msg: str) -> None:
        if self.verbose:
            print(msg)

    def _initialize_index(self) -> None:
        """Every block points at its base-file slot; a missing base file is
        created sparse at its full size (log_storage_manager.py:169-202)."""
        base = self.file_paths[0]
        if not base.exists():
            self._log(f"[LogStorage] Creating new base file at {base}")
            with open(base, "wb") as f:
                if self.num_blocks * self.bytes_per_block > 0:
                    f.seek(self.num_blocks * self.bytes_per_block - 1)
                    f.write(b"\0")
        else:
            self._log(f"[LogStorage] Loaded base file with {self.num_blocks} blocks")
        for b in range(self.num_blocks):
            self.index[b] = BlockLocation(0, b * self.bytes_per_block, self.bytes_per_block, 0)

    def _fd(self, file_id: int) -> int:
        with self._fd_lock:
            fd = self._fds.get(file_id)
            if fd is None:
                fd = os.open(self.file_paths[file_id], os.O_RDONLY)
                self._fds[file_id] = fd
            return fd

    def _grouped(self, block_ids: Iterable[int]) -> List[Tuple[int, List[Tuple[int, BlockLocation]]]]:
        """(file id, [(block, location)] by offset) in order of first appearance
        (log_storage_manager.py:226-252)."""
        groups: Dict[int, List[Tuple[int, BlockLocation]]] = {}
        with self.index_lock:
            for b in block_ids:
                b = int(b)
                if b not in self.index:
                    raise ValueError(f"Block {b} not in index")
                loc = self.index[b]
                groups.setdefault(loc.file_id, []).append((b, loc))
        out = []
        for fid, items in groups.items():
            items.sort(key=lambda it: it[1].offset)
            out.append((fid, items))
        return out

    def read_blocks(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        """{block: (rows, point_dim) fp32} of fresh CPU tensors, read grouped
        by file and by ascending offset (log_storage_manager.py:204-278)."""
        if not block_ids:
            return {}
        result: Dict[int, torch.Tensor] = {}
        for fid, items in self._grouped(block_ids):
            fd = self._fd(fid)
            for b, loc in items:
                if loc.size <= 0:
                    print(f"[LogStorage] WARNING: block {b} points to an empty patch record; "
                          "falling back to base file")
                    result[b] = self._read_base_block(b)
                    continue
                data = np.frombuffer(os.pread(fd, loc.size, loc.offset), dtype=np.float32).copy()
                n = data.size // self.point_dim
                if n <= 0:
                    print(f"[LogStorage] WARNING: block {b} read as empty from "
                          f"{self.file_paths[fid]}; falling back to base file")
                    result[b] = self._read_base_block(b)
                else:
                    result[b] = torch.from_numpy(data).reshape(n, self.point_dim)
            self.stats["reads"] += len(items)
        return result

    def _read_base_block(self, block_id: int) -> torch.Tensor:
        data = np.frombuffer(os.pread(self._fd(0), self.bytes_per_block,
                                      int(block_id) * self.bytes_per_block),
                             dtype=np.float32).copy()
        n = data.size // self.point_dim
        if n <= 0:
            raise RuntimeError(f"Base segment returned empty data for block {block_id}")
        return torch.from_numpy(data).reshape(n, self.point_dim)

    def read_blocks_into(self, block_ids: List[int], dest: Dict[int, torch.Tensor]) -> Dict[int, int]:
        """Reads each block straight into `dest[block]` (a contiguous CPU fp32
        tensor of at least the stored rows, e.g. a page-locked slab entry);
        returns {block: rows read} in the order `read_blocks` uses. Reads of
        distinct blocks run on `read_threads` threads."""
        order: List[Tuple[int, int, BlockLocation]] = []
        for fid, items in self._grouped(block_ids):
            order += [(fid, b, loc) for b, loc in items]

        def one(job) -> int:
            fid, b, loc = job
            if loc.size <= 0:
                loc = BlockLocation(0, b * self.bytes_per_block, self.bytes_per_block, loc.version)
                fid = 0
            view = _byte_view(dest[b])
            if loc.size > len(view):
                raise ValueError(f"Block {b}: stored record of {loc.size} B exceeds the "
                                 f"destination of {len(view)} B")
            got = os.preadv(self._fd(fid), [view[:loc.size]], loc.offset)
            if got != loc.size:
                raise OSError(f"Short read of block {b}: {got} of {loc.size} B")
            return loc.size // self.bytes_per_point

        if len(order) > 1 and self.read_threads > 1:
            from concurrent.futures import ThreadPoolExecutor

            with ThreadPoolExecutor(min(self.read_threads, len(order))) as pool:
                rows = list(pool.map(one, order))
        else:
            rows = [one(j) for j in order]
        self.stats["reads"] += len(order)
        return {b: r for (_, b, _), r in zip(order, rows)}

    def write_patch(self, block_dict: Dict[int, torch.Tensor]) -> int:
        """Appends the blocks (ascending id) to a new patch file, fsyncs it, then
        points the index at it; returns the patch id or -1 when nothing valid
        was given (log_storage_manager.py:293-395)."""
        if not block_dict:
            return -1
        valid: Dict[int, torch.Tensor] = {}
        for b, t in block_dict.items():
            if t is None or t.numel() == 0:
                print(f"[LogStorage] WARNING: skip empty dirty block {b}")
                continue
            if t.dim() != 2 or t.shape[1] != self.point_dim:
                raise ValueError(f"Invalid dirty block {b} shape {tuple(t.shape)}; "
                                 f"expected (*, {self.point_dim})")
            if t.shape[0] > self.block_size:
                raise ValueError(f"Invalid dirty block {b} rows {t.shape[0]}; "
                                 f"expected at most {self.block_size}")
            valid[int(b)] = t
        if not valid:
            print("[LogStorage] Skipped patch creation: no non-empty dirty blocks")
            return -1
        with self._write_lock:
            with self.patch_counter_lock:
                patch_id = self.next_patch_id
                self.next_patch_id += 1
            path = self.storage_dir / f"patch_{patch_id:06d}_{int(time.time() * 1e6)}.bin"
            offset = 0
            locations: Dict[int, BlockLocation] = {}
            fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o644)
            try:
                for b in sorted(valid):
                    t = valid[b]
                    if t.device.type != "cpu":
                        t = t.cpu()
                    t = t.to(torch.float32).contiguous()
                    view = _byte_view(t)
                    done = 0
                    while done < len(view):
                        done += os.write(fd, view[done:])
                    with self.index_lock:
                        old = self.index[b].version if b in self.index else 0
                    locations[b] = BlockLocation(patch_id, offset, len(view), old + 1)
                    offset += len(view)
                os.fsync(fd)
            except BaseException:
                os.close(fd)
                path.unlink(missing_ok=True)
                raise
            os.close(fd)
            with self.index_lock:
                self.file_paths[patch_id] = path
                self.index.update(locations)
            self.stats["writes"] += len(valid)
            self.stats["patches_created"] += 1
            self._log(f"[LogStorage] Created patch {patch_id} with {len(valid)} blocks "
                      f"({offset / 1024 / 1024:.2f} MB)")
            return patch_id

    def get_stats(self) -> Dict:
        """Statistics with the reference's keys (log_storage_manager.py:747-764)."""
        with self.index_lock:
            paths = dict(self.file_paths)
            live = [(b, loc) for b, loc in self.index.items() if loc.file_id != 0]
        patch_paths = {fid: p for fid, p in paths.items() if fid != 0}
        patch_bytes = sum(p.stat().st_size for p in patch_paths.values() if p.exists())
        live_bytes = sum(loc.size for _, loc in live)
        total = sum(p.stat().st_size for p in paths.values() if p.exists())
        import shutil

        return {
            **self.stats,
            "total_files": len(paths),
            "total_size_mb": total / 1024 / 1024,
            "num_patches": len(patch_paths),
            "patch_size_mb": patch_bytes / 1024 / 1024,
            "live_patch_blocks": len(live),
            "live_patch_size_mb": live_bytes / 1024 / 1024,
            "stale_patch_size_mb": max(0, patch_bytes - live_bytes) / 1024 / 1024,
            "free_space_gb": shutil.disk_usage(self.storage_dir).free / (1024 ** 3),
        }

    def close(self) -> None:
        with self._fd_lock:
            for fd in self._fds.values():
                os.close(fd)
            self._fds.clear()


# ---------------------------------------------------------------------------
# RAM block cache (tiered_cache_manager.py) on a page-locked slab
# ---------------------------------------------------------------------------
def _slab(capacity: int, block_size: int, point_dim: int, pin: Optional[bool]) -> torch.Tensor:
    shape = (max(1, capacity), block_size, point_dim)
    if pin is None:
        pin = torch.cuda.is_available()
    if pin:
        return torch.empty(shape, dtype=torch.float32, pin_memory=True)
    return torch.empty(shape, dtype=torch.float32)


class PinnedBlockCache:
    """RAM cache and write buffer of blocks with the reference's LRU, dirty
    and version semantics, stored in one page-locked slab
    (tiered_cache_manager.py:21-175).

    `capacity_blocks` is the number of slab entries (default: the blocks
    `max_ram_gb` holds, plus 25 % for blocks waiting in the flushing buffer).
    The eviction rule is the reference's: after an upsert or a prefetch, if
    the cached blocks exceed `eviction_threshold` of `max_ram_gb`, the least
    recently used 20 % leave (dirty ones through the flushing buffer and the
    block log). When a new block finds no free entry, the least recently
    used clean block is evicted early. When every entry is dirty, flushing or
    waiting to be written, the caller waits (up to `slab_wait_s`) for queued
    flushes to return entries, and RuntimeError if none comes back.

    Writes of one block reach the block log in the order they were queued: a
    synchronous write (flush queue full, flush_all_dirty) first waits for the
    queued ones, since the log keeps whichever write of a block came last.

    An entry is referenced by the cache, by the flushing buffer and by each
    queued flush job that writes it; it returns to the free list when the
    last reference is dropped.
    """

    def __init__(self, storage_manager, max_ram_gb: float = 16.0, block_size: int = 4096,
                 point_dim: int = 59, prefetch_distance: int = 5,
                 eviction_threshold: float = 0.8, verbose: bool = True,
                 capacity_blocks: Optional[int] = None, pin_memory: Optional[bool] = None,
                 slab_wait_s: float = 120.0):
        self.storage = storage_manager
        self.max_ram_bytes = int(max_ram_gb * 1024 * 1024 * 1024)
        self.block_size = int(block_size)
        self.point_dim = int(point_dim)
        self.prefetch_distance = prefetch_distance
        self.eviction_threshold = eviction_threshold
        self.verbose = bool(verbose)
        self.bytes_per_block = self.block_size * self.point_dim * 4
        if capacity_blocks is None:
            fit = -(-self.max_ram_bytes // self.bytes_per_block)
            capacity_blocks = fit + max(1, fit // 4)
        self.capacity_blocks = int(capacity_blocks)
        self.slab = _slab(self.capacity_blocks, self.block_size, self.point_dim, pin_memory)
        self._entry_bytes = self.block_size * self.point_dim * 4
        self._free: List[int] = list(range(self.capacity_blocks - 1, -1, -1))
        self._refs = np.zeros(self.capacity_blocks, np.int32)
        self._dma_reads: Dict[int, object] = {}  # entry -> CUDA event of its last DMA read
        self._cache_entry: Dict[int, int] = {}   # block -> entry of cache_data[block]
        self._flush_entry: Dict[int, int] = {}   # block -> entry of flushing_buffer[block]

        self.cache_data: "OrderedDict[int, torch.Tensor]" = OrderedDict()
        self.dirty_set: Set[int] = set()
        self.block_versions: Dict[int, int] = {}
        self.cache_lock = threading.RLock()
        self._entry_freed = threading.Condition(self.cache_lock)
        self.slab_wait_s = float(slab_wait_s)
        self.flushing_buffer: Dict[int, Tuple[torch.Tensor, float, int]] = {}
        self.flushing_lock = threading.RLock()
        self.flush_queue: Queue = Queue(maxsize=128)
        self.future_prefetch_queue: Queue = Queue(maxsize=64)
        self.future_pending: Set[int] = set()
        self.future_lock = threading.RLock()
        self.inflight_reads: Dict[int, threading.Event] = {}
        self.inflight_lock = threading.RLock()
        self.prefetch_history: Set[int] = set()
        self.stats = {k: 0 for k in (
            "cache_hits", "cache_misses", "evictions", "flushes", "prefetches", "syncs",
            "async_flush_requests", "flush_queue_drops", "async_flush_jobs", "async_flush_blocks",
            "sync_flush_jobs", "sync_flush_blocks", "urgent_prefetch_calls",
            "urgent_prefetch_blocks", "urgent_prefetch_miss_blocks", "future_prefetch_submitted",
            "future_prefetch_skipped", "future_prefetch_dropped", "future_prefetch_jobs",
            "future_prefetch_blocks", "future_prefetch_errors", "future_prefetch_reserved",
            "inflight_wait_blocks", "inflight_fallback_blocks", "direct_writeback_blocks")}
        for k in ("async_flush_time", "sync_flush_time", "urgent_prefetch_time",
                  "future_prefetch_time", "inflight_wait_time"):
            self.stats[k] = 0.0
        self.flush_running = True
        self.flush_thread = threading.Thread(target=self._flush_worker, daemon=True)
        self.flush_thread.start()
        self.future_prefetch_running = True
        self.future_prefetch_thread = threading.Thread(target=self._future_prefetch_worker,
                                                       daemon=True)
        self.future_prefetch_thread.start()

    def _log(self, msg: str) -> None:
        if self.verbose:
            print(msg)

    # -- slab entries --------------------------------------------------------
    def _view(self, entry: int, rows: int) -> torch.Tensor:
        return self.slab[entry, :rows]

    def _release(self, entry: int) -> None:
        """Drops one reference (caller holds cache_lock)."""
        self._refs[entry] -= 1
        if self._refs[entry] == 0:
            self._free.append(entry)
            self._entry_freed.notify_all()

    def _take_entry(self) -> int:
        """A free entry (caller holds cache_lock), after any DMA still
        reading it has finished."""
        if not self._free:
            self._make_room()
        e = self._free.pop()
        ev = self._dma_reads.pop(e, None)
        if ev is not None:
            ev.synchronize()
        self._refs[e] = 1
        return e

    def _make_room(self) -> None:
        """Frees an entry (caller holds cache_lock): evicts the least recently
        used clean block, else waits for queued flushes to return entries."""
        deadline = None
        while not self._free:
            for b in list(self.cache_data.keys()):
                if b not in self.dirty_set and self._refs[self._cache_entry[b]] == 1:
                    self.cache_data.pop(b)
                    self._release(self._cache_entry.pop(b))
                    self.stats["evictions"] += 1
                    return
            with self.flushing_lock:
                pending = bool(self.flushing_buffer) or self.flush_queue.unfinished_tasks > 0
            now = time.monotonic()
            deadline = now + self.slab_wait_s if deadline is None else deadline
            if not pending or now >= deadline:
                raise RuntimeError(f"[TieredCache] slab of {self.capacity_blocks} entries is full "
                                   "(every entry dirty, flushing or shared)")
            # releases cache_lock while waiting, so the flush worker can finish
            self._entry_freed.wait(timeout=min(0.5, deadline - now))

    def _store(self, block_id: int, src: Optional[torch.Tensor], rows: int) -> torch.Tensor:
        """Puts a new entry for block_id (copy of src when given) at the MRU end
        of the cache, replacing any previous entry (caller holds cache_lock)."""
        e = self._take_entry()
        view = self._view(e, rows)
        if src is not None:
            view.copy_(src)
        old = self._cache_entry.pop(block_id, None)
        if old is not None:
            self._release(old)
        self._cache_entry[block_id] = e
        self.cache_data[block_id] = view
        self.cache_data.move_to_end(block_id)
        return view

    def note_dma_reads(self, block_ids: Iterable[int], event) -> None:
        """Records that a DMA reads these blocks' entries until `event`: their
        entries are not rewritten before it has completed."""
        with self.cache_lock:
            for b in block_ids:
                e = self._cache_entry.get(int(b))
                if e is not None:
                    self._dma_reads[e] = event

    def block_host_pointers(self, block_ids) -> Tuple[np.ndarray, np.ndarray]:
        """(host addresses, rows) of cached blocks, for one DMA per block;
        blocks not cached are fetched first (prefetch)."""
        ids = [int(b) for b in block_ids]
        views = self.prefetch(ids)
        ptrs = np.empty(len(ids), np.int64)
        rows = np.empty(len(ids), np.int64)
        for i, b in enumerate(ids):
            view = views.get(b)
            if view is None:
                raise KeyError(f"BlockReader omitted blocks; first missing={[b]}")
            ptrs[i] = view.data_ptr()
            rows[i] = view.shape[0]
        return ptrs, rows

    # -- lookups and single-flight reads -------------------------------------
    def _lookup_cached_or_flushing(self, block_id: int, promote_flushing: bool = False):
        with self.cache_lock:
            t = self.cache_data.get(block_id)
            if t is not None:
                self.cache_data.move_to_end(block_id)
                return t, "cache"
        with self.flushing_lock:
            entry = self.flushing_buffer.get(block_id)
        if entry is None:
            return None, None
        t = entry[0]
        if promote_flushing:
            with self.cache_lock:
                cached = self.cache_data.get(block_id)
                if cached is not None:
                    self.cache_data.move_to_end(block_id)
                    return cached, "cache"
                with self.flushing_lock:
                    e = self._flush_entry.get(block_id)
                if e is not None:
                    self._refs[e] += 1
                    self._cache_entry[block_id] = e
                self.cache_data[block_id] = t
                self.cache_data.move_to_end(block_id)
        return t, "flushing"

    def _reserve_inflight_read(self, block_id: int) -> Tuple[threading.Event, bool]:
        with self.inflight_lock:
            ev = self.inflight_reads.get(block_id)
            if ev is not None:
                return ev, False
            ev = threading.Event()
            self.inflight_reads[block_id] = ev
            return ev, True

    def _complete_inflight_reads(self, block_ids: Iterable[int]) -> None:
        events = []
        with self.inflight_lock:
            for b in block_ids:
                ev = self.inflight_reads.pop(int(b), None)
                if ev is not None:
                    events.append(ev)
        for ev in events:
            ev.set()

    def _wait_for_inflight_read(self, event: threading.Event) -> None:
        t0 = time.time()
        event.wait()
        self.stats["inflight_wait_blocks"] += 1
        self.stats["inflight_wait_time"] += time.time() - t0

    def _load_from_storage(self, block_ids: List[int], only_missing: bool = False) -> List[int]:
        """Reads blocks from the storage into new entries and caches them in
        the storage's order; returns the blocks cached."""
        into = getattr(self.storage, "read_blocks_into", None)
        loaded: List[int] = []
        if callable(into):
            with self.cache_lock:
                dest = {b: self._view(self._take_entry(), self.block_size) for b in block_ids}
            try:
                rows = into(block_ids, dest)
            except BaseException:
                with self.cache_lock:
                    for v in dest.values():
                        self._release(self._entry_of(v))
                raise
            with self.cache_lock:
                for b, n in rows.items():
                    e = self._entry_of(dest.pop(b))
                    if only_missing and (b in self.cache_data or self._in_flushing(b)):
                        self._release(e)
                        continue
                    old = self._cache_entry.pop(b, None)
                    if old is not None:
                        self._release(old)
                    self._cache_entry[b] = e
                    self.cache_data[b] = self._view(e, n)
                    self.cache_data.move_to_end(b)
                    loaded.append(b)
                for v in dest.values():
                    self._release(self._entry_of(v))
            return loaded
        tensors = self.storage.read_blocks(block_ids)
        with self.cache_lock:
            for b, t in tensors.items():
                if only_missing and (b in self.cache_data or self._in_flushing(b)):
                    continue
                self._store(int(b), t, int(t.shape[0]))
                loaded.append(int(b))
        return loaded

    def _in_flushing(self, block_id: int) -> bool:
        with self.flushing_lock:
            return block_id in self.flushing_buffer

    def _entry_of(self, view: torch.Tensor) -> int:
        return (view.data_ptr() - self.slab.data_ptr()) // self._entry_bytes

    def _read_claimed_blocks(self, block_ids: List[int], result: Dict[int, torch.Tensor],
                             cache_hits: List[int]) -> Tuple[int, float]:
        if not block_ids:
            return 0, 0.0
        to_read, resolved = [], []
        for b in block_ids:
            t, source = self._lookup_cached_or_flushing(b)
            if t is not None:
                result[b] = t
                cache_hits.append(b)
                resolved.append(b)
            else:
                to_read.append(b)
        if resolved:
            self._complete_inflight_reads(resolved)
        if not to_read:
            return 0, 0.0
        t0 = time.time()
        try:
            loaded = self._load_from_storage(to_read)
            with self.cache_lock:
                for b in loaded:
                    result[b] = self.cache_data[b]
            return len(to_read), time.time() - t0
        finally:
            self._complete_inflight_reads(to_read)

    # -- flushing ------------------------------------------------------------
    def _to_flushing(self, block_id: int, view: torch.Tensor, entry: Optional[int],
                     version: int, now: float) -> None:
        """flushing_buffer[block_id] = view (caller holds flushing_lock); the
        flushing buffer takes one reference on the entry."""
        old = self._flush_entry.pop(block_id, None)
        if old is not None:
            self._release(old)
        if entry is not None:
            self._flush_entry[block_id] = entry
        self.flushing_buffer[block_id] = (view, now, version)

    def _submit_flush(self, dirty_blocks: Dict[int, torch.Tensor], versions: Dict[int, int],
                      reason: str) -> None:
        """Hands a flush job to the worker (synchronously when its queue is
        full); the job holds a reference on each entry it writes."""
        if not dirty_blocks:
            return
        with self.cache_lock:
            for t in dirty_blocks.values():
                self._refs[self._entry_of(t)] += 1
        if not self._enqueue_dirty_flush(dirty_blocks, versions, reason):
            self._flush_in_order(dirty_blocks, versions)

    def _flush_in_order(self, dirty_blocks: Dict[int, torch.Tensor],
                        versions: Dict[int, int]) -> None:
        """Synchronous write after every queued flush job: a queued job may
        hold an older version of one of these blocks, and the block log keeps
        whichever write of a block came last. The caller holds no lock."""
        if threading.current_thread() is not self.flush_thread:
            self.flush_queue.join()
        self._flush_dirty_blocks(dirty_blocks, block_versions=versions, mode="sync")

    def _flush_dirty_blocks(self, dirty_blocks: Dict[int, torch.Tensor],
                            block_versions: Optional[Dict[int, int]] = None,
                            mode: str = "async") -> None:
        """Writes a flush job and drops its entry references."""
        if not dirty_blocks:
            return
        try:
            self._write_flush(dirty_blocks, block_versions or {}, mode)
        finally:
            with self.cache_lock:
                for t in dirty_blocks.values():
                    self._release(self._entry_of(t))

    def _write_flush(self, dirty_blocks: Dict[int, torch.Tensor], block_versions: Dict[int, int],
                     mode: str) -> None:
        t0 = time.time()
        try:
            self.storage.write_patch(dirty_blocks)
            elapsed = time.time() - t0
            with self.cache_lock, self.flushing_lock:
                for b in dirty_blocks:
                    flushed = block_versions.get(b)
                    cur = self.flushing_buffer.get(b)
                    if cur is not None and (flushed is None or cur[2] <= flushed):
                        self.flushing_buffer.pop(b, None)
                        e = self._flush_entry.pop(b, None)
                        if e is not None:
                            self._release(e)
                for b in dirty_blocks:
                    flushed = block_versions.get(b)
                    if flushed is None or self.block_versions.get(b, 0) == flushed:
                        self.dirty_set.discard(b)
            self.stats["flushes"] += 1
            key = "async" if mode == "async" else "sync"
            self.stats[f"{key}_flush_jobs"] += 1
            self.stats[f"{key}_flush_blocks"] += len(dirty_blocks)
            self.stats[f"{key}_flush_time"] += elapsed
        except Exception as exc:
            print(f"[TieredCache] ERROR during SSD write: {exc}")
            with self.cache_lock, self.flushing_lock:
                for b, t in dirty_blocks.items():
                    if b not in self.cache_data:
                        e = self._entry_of(t)
                        self._refs[e] += 1
                        self._cache_entry[b] = e
                        self.cache_data[b] = t
                        self.cache_data.move_to_end(b)
                    self.dirty_set.add(b)
                    self.flushing_buffer.pop(b, None)
                    e = self._flush_entry.pop(b, None)
                    if e is not None:
                        self._release(e)
            raise

    def _enqueue_dirty_flush(self, dirty_blocks, block_versions=None, reason="background") -> bool:
        if not dirty_blocks:
            return True
        try:
            self.flush_queue.put_nowait((reason, dirty_blocks, block_versions or {}))
            self.stats["async_flush_requests"] += 1
            return True
        except Full:
            self.stats["flush_queue_drops"] += 1
            print(f"[TieredCache] Flush queue full; falling back to synchronous write for "
                  f"{len(dirty_blocks)} blocks (after the queued ones)")
            return False

    def _flush_worker(self) -> None:
        while self.flush_running or not self.flush_queue.empty():
            try:
                reason, blocks, versions = self.flush_queue.get(timeout=0.1)
            except Empty:
                continue
            try:
                self._flush_dirty_blocks(blocks, block_versions=versions, mode="async")
            except Exception as exc:
                print(f"[TieredCache] Flush worker error ({reason}): {exc}")
            finally:
                self.flush_queue.task_done()

    def _future_prefetch_worker(self) -> None:
        while self.future_prefetch_running or not self.future_prefetch_queue.empty():
            try:
                block_ids = self.future_prefetch_queue.get(timeout=0.1)
            except Empty:
                continue
            block_ids = [int(b) for b in block_ids]
            t0 = time.time()
            try:
                to_load = [b for b in block_ids
                           if self._lookup_cached_or_flushing(b, promote_flushing=True)[0] is None]
                count = len(self._load_from_storage(to_load, only_missing=True)) if to_load else 0
                self.stats["future_prefetch_jobs"] += 1
                self.stats["future_prefetch_blocks"] += count
                self.stats["future_prefetch_time"] += time.time() - t0
                if count:
                    self.stats["prefetches"] += count
                self._maybe_evict()
            except Exception as exc:
                self.stats["future_prefetch_errors"] += 1
                print(f"[TieredCache] Future prefetch worker error: {exc}")
            finally:
                self._complete_inflight_reads(block_ids)
                with self.future_lock:
                    for b in block_ids:
                        self.future_pending.discard(b)
                self.future_prefetch_queue.task_done()

    # -- writes into the cache -----------------------------------------------
    def _is_valid_block_tensor(self, block_id, tensor, context: str) -> bool:
        if tensor is None or tensor.numel() == 0:
            print(f"[TieredCache] WARNING: skip empty block {block_id} during {context}")
            return False
        if tensor.dim() != 2 or tensor.shape[1] != self.point_dim:
            raise ValueError(f"Invalid block {block_id} shape {tuple(tensor.shape)} during "
                             f"{context}; expected (*, {self.point_dim})")
        if tensor.shape[0] > self.block_size:
            raise ValueError(f"Invalid block {block_id} rows {tensor.shape[0]} during {context}; "
                             f"expected at most {self.block_size}")
        return True

    def _mark_dirty(self, block_id: int) -> None:
        self.block_versions[block_id] = self.block_versions.get(block_id, 0) + 1
        self.dirty_set.add(block_id)

    def upsert_dirty_blocks(self, block_tensors: Dict[int, torch.Tensor], clone: bool = False) -> int:
        """Copies the blocks into the cache and marks them dirty
        (tiered_cache_manager.py:499-522); every block gets its own entry, so
        `clone` makes no difference."""
        if not block_tensors:
            return 0
        staged = 0
        with self.cache_lock:
            for b, t in block_tensors.items():
                if not self._is_valid_block_tensor(b, t, "upsert_dirty_blocks"):
                    continue
                self._store(int(b), t, int(t.shape[0]))
                self._mark_dirty(int(b))
                staged += 1
        self._maybe_evict()
        return staged

    def upsert_dirty_block_batch(self, block_tensors: Dict[int, torch.Tensor]) -> int:
        """Owns a copy of a staged write-back batch (tiered_cache_manager.py:524-599);
        the entries of one batch are views of the cache's single slab."""
        if not block_tensors:
            return 0
        items = [(int(b), t) for b, t in block_tensors.items()
                 if self._is_valid_block_tensor(b, t, "upsert_dirty_block_batch")]
        if not items:
            return 0
        with self.cache_lock:
            for b, t in items:
                self._store(b, t, int(t.shape[0]))
                self._mark_dirty(b)
        self._maybe_evict()
        return len(items)

    def reserve_writeback(self, plans: Sequence[Tuple[int, int]]) -> List[torch.Tensor]:
        """Fresh entries for a write-back batch [(block, rows)] that a DMA fills;
        publish them with `commit_writeback` once it has landed (or return
        them with `abort_writeback`)."""
        with self.cache_lock:
            out = []
            for b, rows in plans:
                if not (0 < int(rows) <= self.block_size):
                    raise ValueError(f"Invalid block {b} rows {rows} during reserve_writeback; "
                                     f"expected 1..{self.block_size}")
                out.append(self._view(self._take_entry(), int(rows)))
            return out

    def commit_writeback(self, plans: Sequence[Tuple[int, int]],
                         views: Sequence[torch.Tensor]) -> int:
        """Publishes filled write-back entries: each block's cached copy becomes
        its entry, dirty, version + 1 (the state `upsert_dirty_block_batch`
        leaves)."""
        with self.cache_lock:
            for (b, _), v in zip(plans, views):
                b = int(b)
                old = self._cache_entry.pop(b, None)
                if old is not None:
                    self._release(old)
                self._cache_entry[b] = self._entry_of(v)
                self.cache_data[b] = v
                self.cache_data.move_to_end(b)
                self._mark_dirty(b)
            self.stats["direct_writeback_blocks"] += len(plans)
        self._maybe_evict()
        return len(plans)

    def abort_writeback(self, views: Sequence[torch.Tensor]) -> None:
        with self.cache_lock:
            for v in views:
                self._release(self._entry_of(v))

    def submit_dirty_blocks(self, block_ids: List[int], clone: bool = True,
                            reason: str = "paper_writeback") -> int:
        """Queues dirty cached blocks for the block log (tiered_cache_manager.py:601-636)."""
        if not block_ids:
            return 0
        blocks: Dict[int, torch.Tensor] = {}
        versions: Dict[int, int] = {}
        entries: Dict[int, int] = {}
        with self.cache_lock:
            for b in block_ids:
                if b not in self.cache_data or b not in self.dirty_set:
                    continue
                t = self.cache_data[b]
                if not self._is_valid_block_tensor(b, t, "submit_dirty_blocks"):
                    self.dirty_set.discard(b)
                    continue
                if clone:
                    # a private copy: later upserts cannot race with its write
                    e = self._take_entry()
                    view = self._view(e, t.shape[0])
                    view.copy_(t)
                else:
                    e = self._cache_entry[b]
                    self._refs[e] += 1
                    view = t
                blocks[b], entries[b] = view, e
                versions[b] = self.block_versions.get(b, 0)
        if not blocks:
            return 0
        with self.cache_lock, self.flushing_lock:
            # the job's references first: a newer flushing version below may
            # drop the flushing reference of an entry the job still writes
            for view in blocks.values():
                self._refs[self._entry_of(view)] += 1
            now = time.time()
            for b, view in blocks.items():
                existing = self.flushing_buffer.get(b)
                if existing is None or existing[2] <= versions[b]:
                    self._to_flushing(b, view, entries[b], versions[b], now)
                else:
                    self._release(entries[b])
        if not self._enqueue_dirty_flush(blocks, versions, reason):
            self._flush_in_order(blocks, versions)
        return len(blocks)

    # -- reads ---------------------------------------------------------------
    def prefetch(self, needed_block_ids: List[int],
                 future_block_ids: Optional[List[int]] = None) -> Dict[int, torch.Tensor]:
        """{block: cached view} for the needed blocks: cache, then flushing
        buffer, then a read another caller has in flight, then the block log
        (tiered_cache_manager.py:637-732)."""
        result: Dict[int, torch.Tensor] = {}
        cache_hits: List[int] = []
        read_ids: List[int] = []
        waits = []
        seen: Set[int] = set()
        self.stats["urgent_prefetch_calls"] += 1
        for raw in needed_block_ids:
            b = int(raw)
            if b in seen:
                continue
            seen.add(b)
            t, source = self._lookup_cached_or_flushing(b)
            if t is not None:
                result[b] = t
                cache_hits.append(b)
                continue
            ev, claimed = self._reserve_inflight_read(b)
            if claimed:
                read_ids.append(b)
            else:
                waits.append((b, ev))
        reads, read_time = self._read_claimed_blocks(read_ids, result, cache_hits)
        while waits:
            fallback, again = [], []
            for b, ev in waits:
                self._wait_for_inflight_read(ev)
                t, source = self._lookup_cached_or_flushing(b)
                if t is not None:
                    result[b] = t
                    cache_hits.append(b)
                    continue
                ev2, claimed = self._reserve_inflight_read(b)
                if claimed:
                    fallback.append(b)
                    self.stats["inflight_fallback_blocks"] += 1
                else:
                    again.append((b, ev2))
            n, dt = self._read_claimed_blocks(fallback, result, cache_hits)
            reads += n
            read_time += dt
            waits = again
        self.stats["urgent_prefetch_blocks"] += reads
        self.stats["urgent_prefetch_miss_blocks"] += reads
        self.stats["urgent_prefetch_time"] += read_time
        self.stats["cache_hits"] += len(cache_hits)
        self.stats["cache_misses"] += reads
        self._maybe_evict()
        return result

    def prefetch_future(self, block_ids: List[int]) -> int:
        """Queues not-yet-cached blocks for the background reader
        (tiered_cache_manager.py:734-783)."""
        to_prefetch, skipped = [], 0
        with self.cache_lock:
            for b in sorted(set(int(x) for x in block_ids)):
                if b in self.cache_data:
                    self.cache_data.move_to_end(b)
                    skipped += 1
                    continue
                if self._in_flushing(b):
                    self._lookup_cached_or_flushing(b, promote_flushing=True)
                    skipped += 1
                    continue
                with self.future_lock:
                    if b in self.future_pending:
                        skipped += 1
                        continue
                    _, claimed = self._reserve_inflight_read(b)
                    if not claimed:
                        skipped += 1
                        continue
                    self.future_pending.add(b)
                to_prefetch.append(b)
        self.stats["future_prefetch_skipped"] += skipped
        if not to_prefetch:
            return 0
        try:
            self.future_prefetch_queue.put_nowait(to_prefetch)
            self.stats["future_prefetch_submitted"] += len(to_prefetch)
            self.stats["future_prefetch_reserved"] += len(to_prefetch)
            return len(to_prefetch)
        except Full:
            self._complete_inflight_reads(to_prefetch)
            with self.future_lock:
                for b in to_prefetch:
                    self.future_pending.discard(b)
            self.stats["future_prefetch_dropped"] += len(to_prefetch)
            print(f"[TieredCache] Future prefetch queue full; dropped {len(to_prefetch)} blocks")
            return 0

    # -- eviction ------------------------------------------------------------
    def _get_ram_usage(self) -> int:
        with self.cache_lock:
            return len(self.cache_data) * self.bytes_per_block

    def _maybe_evict(self) -> None:
        if self._get_ram_usage() > self.max_ram_bytes * self.eviction_threshold:
            self.evict_and_flush(num_blocks=int(len(self.cache_data) * 0.2))

    def evict_and_flush(self, num_blocks: Optional[int] = None) -> None:
        """Evicts the least recently used blocks; dirty ones go through the
        flushing buffer to the block log (tiered_cache_manager.py:800-859)."""
        if num_blocks is None:
            num_blocks = max(1, int(len(self.cache_data) * 0.2))
        victims: List[int] = []
        dirty: Dict[int, torch.Tensor] = {}
        versions: Dict[int, int] = {}
        with self.cache_lock:
            for _ in range(min(num_blocks, len(self.cache_data))):
                if not self.cache_data:
                    break
                b, t = self.cache_data.popitem(last=False)
                e = self._cache_entry.pop(b)
                victims.append(b)
                if b in self.dirty_set:
                    if not self._is_valid_block_tensor(b, t, "evict_and_flush"):
                        self.dirty_set.discard(b)
                        self._release(e)
                        continue
                    dirty[b] = t
                    versions[b] = self.block_versions.get(b, 0)
                    with self.flushing_lock:
                        # the cache's reference on the entry moves to the flushing buffer
                        self._refs[e] += 1
                        self._to_flushing(b, t, e, versions[b], time.time())
                self._release(e)
        self._submit_flush(dirty, versions, "evict")
        self.stats["evictions"] += len(victims)
        if victims:
            self._log(f"[TieredCache] Evicted {len(victims)} blocks ({len(dirty)} dirty)")

    def flush_all_dirty(self) -> None:
        """Writes every dirty cached block to the block log (tiered_cache_manager.py:861-883)."""
        with self.cache_lock:
            blocks = {b: self.cache_data[b] for b in self.dirty_set if b in self.cache_data}
            versions = {b: self.block_versions.get(b, 0) for b in blocks}
            entries = {b: self._cache_entry[b] for b in blocks}
            if blocks:
                with self.flushing_lock:
                    now = time.time()
                    for b, t in blocks.items():
                        self._refs[entries[b]] += 1
                        self._to_flushing(b, t, entries[b], versions[b], now)
        if blocks:
            self._log(f"[TieredCache] Flushing {len(blocks)} dirty blocks to SSD")
            with self.cache_lock:
                for t in blocks.values():
                    self._refs[self._entry_of(t)] += 1
            self._flush_in_order(blocks, versions)

    def get_stats(self) -> Dict:
        with self.cache_lock:
            size, dirty = len(self.cache_data), len(self.dirty_set)
            ram_mb = self._get_ram_usage() / 1024 / 1024
        with self.flushing_lock:
            flushing = len(self.flushing_buffer)
        with self.future_lock:
            pending = len(self.future_pending)
        with self.inflight_lock:
            inflight = len(self.inflight_reads)
        total = self.stats["cache_hits"] + self.stats["cache_misses"]
        return {
            **self.stats,
            "cache_size": size, "dirty_blocks": dirty, "flushing_blocks": flushing,
            "flush_queue_size": self.flush_queue.qsize(),
            "future_queue_size": self.future_prefetch_queue.qsize(),
            "future_pending_blocks": pending,
            "future_prefetch_queue_size": self.future_prefetch_queue.qsize(),
            "future_prefetch_pending": pending, "inflight_read_blocks": inflight,
            "ram_usage_mb": ram_mb, "hit_rate": self.stats["cache_hits"] / total if total else 0.0,
            "max_ram_mb": self.max_ram_bytes / 1024 / 1024,
            "slab_entries": self.capacity_blocks, "free_entries": len(self._free),
        }

    def drain(self) -> None:
        """Waits until the flush and future-prefetch queues are empty."""
        self.flush_queue.join()
        self.future_prefetch_queue.join()

    def shutdown(self) -> None:
        """Drains the workers and writes every dirty block (tiered_cache_manager.py:923-970)."""
        self.flush_queue.join()
        self.future_prefetch_queue.join()
        self.flush_all_dirty()
        self.future_prefetch_running = False
        self.future_prefetch_thread.join(timeout=5.0)
        self.flush_running = False
        self.flush_thread.join(timeout=5.0)


class CachedBlockReader:
    """BlockReader over a `PinnedBlockCache` (block_reader.py:179-236
    `TieredCacheBlockReader`), plus the page-locked DMA interface the
    materializer uses (`block_host_pointers`, `note_dma_reads`)."""

    layout = BlockLayout.CACHE

    def __init__(self, cache_manager, total_gaussians: int, block_size: int,
                 before_read=None, filter_hint=None):
        if cache_manager is None:
            raise ValueError("TieredCacheBlockReader requires a non-None cache_manager")
        self._cache = cache_manager
        self.total_gaussians = int(total_gaussians)
        self.block_size = int(block_size)
        self.num_blocks = (self.total_gaussians + self.block_size - 1) // self.block_size
        self._before_read = before_read
        self._filter_hint = filter_hint

    def _valid(self, block_ids) -> List[int]:
        return [int(b) for b in block_ids if 0 <= int(b) < self.num_blocks]

    def read_blocks(self, block_ids: List[int]) -> Dict[int, torch.Tensor]:
        valid = self._valid(block_ids)
        if not valid:
            return {}
        if self._before_read is not None:
            self._before_read(valid)
        return self._cache.prefetch(valid)

    def read_batch(self, block_ids: List[int], out: Optional[torch.Tensor] = None):
        valid = self._valid(block_ids)
        return _pack_block_batch(self.read_blocks(valid), valid, self.layout, out)

    def hint_future(self, block_ids: List[int]) -> int:
        valid = self._valid(block_ids)
        if self._filter_hint is not None:
            valid = self._filter_hint(valid)
        if not valid:
            return 0
        return int(self._cache.prefetch_future(valid) or 0)

    def contains_block(self, block_id: int) -> bool:
        return 0 <= int(block_id) < self.num_blocks

    def block_host_pointers(self, block_ids):
        ids = np.asarray(block_ids, dtype=np.int64)
        bad = ids[(ids < 0) | (ids >= self.num_blocks)]
        if bad.size:
            raise KeyError(f"BlockReader omitted blocks; first missing={bad[:8].tolist()}")
        if self._before_read is not None:
            self._before_read(ids.tolist())
        return self._cache.block_host_pointers(ids.tolist())

    def note_dma_reads(self, block_ids, event) -> None:
        self._cache.note_dma_reads(block_ids, event)
