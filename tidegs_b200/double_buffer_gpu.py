"""Double-buffered resident-slot materialization with N+1 prefetch (drop-in for
TideGS's strategies/tide_engine/double_buffer_gpu.py).

Same classes (GPUBuffer, ResidentHandoffResult, DoubleBufferGPUWorkingSet),
methods, worker threads ("tide-nplus1", "tide-resident-plan"), streams,
statistics and block ordering rules as the reference. Device work:

* streamed blocks: one H2D of the packed rows (or, for a PinnedBlockPool, one
  DMA per block straight from the pool), then `tgs_unpack_rows` scatters them
  into the six component arrays and writes their global ids in the same pass
  (reference: Triton unpack :150-209 + id fill :130-148, two launches);
* slot remap / retained-block refresh: `tgs_copy_blocks`, block-granular TMA
  bulk copies (reference: per-element Triton gather :40-128);
* dirty tracking: a bit-packed bitmap with warp-ballot compaction
  (reference: bool bitmap + index_select/nonzero :494-543);
* block-start table / global->local: `tgs_build_block_starts`,
  `tgs_global_to_local(_compact)` (reference :212-256).
"""
from __future__ import annotations

import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib, _ops
from .block_reader import component_columns, layout_code


def _build_block_starts(block_to_local_slice: Dict[int, slice], num_blocks: int,
                        device: torch.device) -> torch.Tensor:
    """[num_blocks] int64: local start of each loaded block, -1 if absent
    (double_buffer_gpu.py:212-234)."""
    return _ops.build_block_starts(
        ((b, s.start) for b, s in block_to_local_slice.items()), num_blocks, device)


def _global_ids_to_local(global_ids: torch.Tensor, block_starts: torch.Tensor,
                         block_size: int) -> torch.Tensor:
    """Global Gaussian ids -> working-set rows, -1 if the block is not loaded
    (double_buffer_gpu.py:237-256)."""
    return _ops.global_to_local(global_ids, block_starts, block_size)


@dataclass
class GPUBuffer:
    """A single GPU buffer holding all Gaussian parameters."""
    xyz: Optional[torch.Tensor] = None
    scaling: Optional[torch.Tensor] = None
    rotation: Optional[torch.Tensor] = None
    opacity: Optional[torch.Tensor] = None
    features_dc: Optional[torch.Tensor] = None
    features_rest: Optional[torch.Tensor] = None
    local_to_global_idx: Optional[torch.Tensor] = None
    _block_starts: Optional[torch.Tensor] = None
    loaded_blocks: List[int] = None
    num_gaussians: int = 0
    filters_local: List[torch.Tensor] = None
    block_to_local_slice: Dict[int, slice] = None
    resident_blocks: List[int] = None
    streamed_blocks: List[int] = None
    evicted_blocks: List[int] = None

    def __post_init__(self):
        if self.loaded_blocks is None:
            self.loaded_blocks = []
        if self.filters_local is None:
            self.filters_local = []
        if self.block_to_local_slice is None:
            self.block_to_local_slice = {}
        if self.resident_blocks is None:
            self.resident_blocks = []
        if self.streamed_blocks is None:
            self.streamed_blocks = []
        if self.evicted_blocks is None:
            self.evicted_blocks = []

    def is_empty(self) -> bool:
        return self.xyz is None

    def components(self) -> Dict[str, torch.Tensor]:
        return {"xyz": self.xyz, "opacity": self.opacity, "scaling": self.scaling,
                "rotation": self.rotation, "features_dc": self.features_dc,
                "features_rest": self.features_rest}

    def clear(self):
        self.xyz = None
        self.scaling = None
        self.rotation = None
        self.opacity = None
        self.features_dc = None
        self.features_rest = None
        self.local_to_global_idx = None
        self._block_starts = None
        self.loaded_blocks = []
        self.filters_local = []
        self.block_to_local_slice = {}
        self.resident_blocks = []
        self.streamed_blocks = []
        self.evicted_blocks = []
        self.num_gaussians = 0


@dataclass(frozen=True)
class ResidentHandoffResult:
    """Outcome of making retained blocks ready for the next activation."""

    ready_blocks: int
    copied_blocks: int


class DoubleBufferGPUWorkingSet:
    """Double-buffered GPU working set manager with N+1 prefetch."""

    def __init__(self, num_total_gaussians: int, block_size: int, device: str = "cuda",
                 verbose: bool = True):
        self.num_total = int(num_total_gaussians)
        self.block_size = int(block_size)
        self.device = _lib.require_cuda(device, "DoubleBufferGPUWorkingSet")
        self.num_blocks = (self.num_total + self.block_size - 1) // self.block_size
        self.verbose = bool(verbose)

        self.buffer_a = GPUBuffer()
        self.buffer_b = GPUBuffer()
        self.active_buffer_idx = 0

        self.prefetch_stream = torch.cuda.Stream(device=self.device)
        self.resident_refresh_stream = torch.cuda.Stream(device=self.device)
        self._unpack_stream = torch.cuda.Stream(device=self.device)
        self.prefetch_complete_event = torch.cuda.Event()
        self.resident_refresh_complete_event: Optional[torch.cuda.Event] = None
        self.prefetch_in_progress = False
        self.prefetch_iteration = -1
        self._prefetch_future: Optional[Future] = None
        self._prefetch_finalized = True
        self._deferred_resident_blocks: List[int] = []
        self._target_layout_ready = threading.Event()
        self._persistent_plan = None
        self._before_persistent_apply = None
        self._prefetch_executor = ThreadPoolExecutor(max_workers=1,
                                                     thread_name_prefix="tide-nplus1")
        self._resident_plan_executor = ThreadPoolExecutor(max_workers=1,
                                                          thread_name_prefix="tide-resident-plan")
        self._resident_plan_future: Optional[Future] = None
        self._executor_shutdown = False
        # two rotating host/device staging slots (double_buffer_gpu.py:748-809)
        self._host_staging_slots: List[Optional[torch.Tensor]] = [None] * 2
        self._gpu_staging_slots: List[Optional[torch.Tensor]] = [None] * 2
        self._host_staging_capacities = [0] * 2
        self._host_staging_events: List[Optional[torch.cuda.Event]] = [None] * 2
        self._next_host_staging_slot = 0
        # Bit-packed dirty bitmap: bit (id & 31) of word id >> 5.
        self._dirty_bitmap = torch.zeros(_ops.bitmap_words(self.num_blocks), dtype=torch.int32,
                                         device=self.device)
        self._err = torch.zeros(4, dtype=torch.int32, device=self.device)

        self.lock = threading.Lock()
        self.stats = {
            "swaps": 0,
            "prefetch_hits": 0,
            "prefetch_misses": 0,
            "total_prefetch_time_ms": 0.0,
            "batched_materializations": 0,
            "batched_h2d_calls": 0,
            "batched_streamed_blocks": 0,
            "batched_resident_blocks": 0,
            "host_staging_bytes": 0,
            "host_staging_pinned": False,
            "dirty_blocks_marked": 0,
            "dirty_blocks_written_back": 0,
            "persistent_slot_updates": 0,
            "persistent_streamed_blocks": 0,
            "persistent_ab_fallbacks": 0,
            "inline_prefetches": 0,
            "persistent_omega_reuses": 0,
            "resident_refresh_blocks": 0,
            "resident_plan_jobs": 0,
            "resident_plan_time_ms": 0.0,
            "direct_block_dma_calls": 0,
        }
        self._log("[DoubleBufferGPU] Initialized with 2 GPU buffers")
        self._log(f"[DoubleBufferGPU] Total Gaussians: {self.num_total:,}")
        self._log(f"[DoubleBufferGPU] Block size: {self.block_size}, Blocks: {self.num_blocks}")

    def _log(self, message: str) -> None:
        if self.verbose:
            print(message)

    @property
    def active_buffer(self) -> GPUBuffer:
        return self.buffer_a if self.active_buffer_idx == 0 else self.buffer_b

    @property
    def loading_buffer(self) -> GPUBuffer:
        return self.buffer_b if self.active_buffer_idx == 0 else self.buffer_a

    @property
    def gpu_xyz(self):
        return self.active_buffer.xyz

    @property
    def gpu_scaling(self):
        return self.active_buffer.scaling

    @property
    def gpu_rotation(self):
        return self.active_buffer.rotation

    @property
    def gpu_opacity(self):
        return self.active_buffer.opacity

    @property
    def gpu_features_dc(self):
        return self.active_buffer.features_dc

    @property
    def gpu_features_rest(self):
        return self.active_buffer.features_rest

    @property
    def local_to_global_idx(self):
        return self.active_buffer.local_to_global_idx

    def global_to_local(self, global_ids: torch.Tensor) -> torch.Tensor:
        buf = self.active_buffer
        if buf._block_starts is None:
            raise RuntimeError(
                "[DoubleBufferGPU] global_to_local called but _block_starts "
                "has not been built yet (buffer is empty or not materialized)"
            )
        return _global_ids_to_local(global_ids, buf._block_starts, self.block_size)

    # ------------------------------------------------------------------
    # Dirty tracking (double_buffer_gpu.py:494-543)
    # ------------------------------------------------------------------
    def _valid_sorted(self, block_ids: List[int]) -> List[int]:
        return sorted(set(int(b) for b in block_ids if 0 <= int(b) < self.num_blocks))

    def mark_dirty_blocks(self, block_ids: List[int]) -> int:
        ids = self._valid_sorted(block_ids)
        if not ids:
            return 0
        with self.lock:
            _ops.dirty_mark(self._dirty_bitmap, ids, True)
            self.stats["dirty_blocks_marked"] += len(ids)
        return len(ids)

    def dirty_blocks_for_eviction(self, evicted_block_ids: List[int]) -> List[int]:
        evicted = self._valid_sorted(evicted_block_ids)
        if not evicted:
            return []
        with self.lock:
            return _ops.dirty_select(self._dirty_bitmap, evicted)

    def dirty_blocks(self) -> List[int]:
        with self.lock:
            return _ops.dirty_list(self._dirty_bitmap, self.num_blocks)

    def mark_blocks_written_back(self, block_ids: List[int]) -> None:
        ids = self._valid_sorted(block_ids)
        if not ids:
            return
        with self.lock:
            _ops.dirty_mark(self._dirty_bitmap, ids, False)
            self.stats["dirty_blocks_written_back"] += len(ids)

    # ------------------------------------------------------------------
    # Resident planner worker (double_buffer_gpu.py:545-570)
    # ------------------------------------------------------------------
    def submit_resident_plan(self, plan_iteration: int, planner: Callable, *args, **kwargs) -> Future:
        previous = self._resident_plan_future
        if previous is not None and not previous.done():
            raise RuntimeError("previous resident plan is still running")

        def _run():
            started = time.perf_counter()
            try:
                return planner(*args, **kwargs)
            finally:
                elapsed_ms = (time.perf_counter() - started) * 1000.0
                with self.lock:
                    self.stats["resident_plan_time_ms"] += elapsed_ms

        with self.lock:
            self.stats["resident_plan_jobs"] += 1
        future = self._resident_plan_executor.submit(_run)
        future.iteration = int(plan_iteration)
        self._resident_plan_future = future
        return future

    # ------------------------------------------------------------------
    # Persistent-slot plan (double_buffer_gpu.py:572-649)
    # ------------------------------------------------------------------
    def _build_persistent_plan(self, next_blocks: List[int], resident_set: set, evicted_set: set,
                               *, allow_resident_copy: bool, defer_resident_copy: bool):
        source = self.active_buffer
        current_blocks = list(source.loaded_blocks)
        if (not allow_resident_copy or not defer_resident_copy or source.is_empty()
                or not current_blocks or len(next_blocks) != len(current_blocks)):
            return None
        current_set = set(map(int, current_blocks))
        next_set = set(map(int, next_blocks))
        keep_set = current_set & next_set
        incoming = sorted(next_set - current_set)
        evicted = current_set - next_set
        if (keep_set != set(map(int, resident_set))
                or evicted != set(map(int, evicted_set))
                or len(incoming) != len(evicted)):
            return None
        slices = source.block_to_local_slice
        if not current_set.issubset(slices.keys()) or any(
                slices[b].stop - slices[b].start != self.block_size for b in current_set):
            return None
        for block_id in incoming:
            if min(self.block_size, self.num_total - int(block_id) * self.block_size) != self.block_size:
                return None
        if int(source.xyz.shape[0]) != len(current_blocks) * self.block_size:
            return None
        # Incoming blocks take the freed slices in ascending slice order.
        free_slices = sorted((source.block_to_local_slice[int(b)] for b in evicted),
                             key=lambda s: int(s.start))
        target_slices = {b: s for b, s in zip(incoming, free_slices)}
        # the full next slot map (next_slices / next_order) is only needed at
        # swap time: persistent_plan_layout() builds it after the DMA is queued
        return {
            "keep_set": keep_set,
            "incoming_blocks": incoming,
            "evicted_blocks": sorted(evicted),
            "target_slices": target_slices,
        }

    def _persistent_plan_layout(self, plan) -> None:
        """Completes a persistent plan with the slot map of the next step:
        kept blocks stay in their slices, incoming ones take the freed ones,
        loaded_blocks in slice order (double_buffer_gpu.py:604-649)."""
        if "next_slices" in plan:
            return
        source = self.active_buffer
        keep_set = plan["keep_set"]
        next_slices = {int(b): source.block_to_local_slice[int(b)] for b in keep_set}
        next_slices.update(plan["target_slices"])
        plan["next_slices"] = next_slices
        plan["next_order"] = [b for b, _ in sorted(next_slices.items(),
                                                   key=lambda it: int(it[1].start))]
        plan["keep_blocks"] = sorted(keep_set)
        plan["block_starts"] = _build_block_starts(next_slices, self.num_blocks, self.device)

    @property
    def loaded_blocks(self) -> List[int]:
        return self.active_buffer.loaded_blocks

    @property
    def filters_local(self) -> List[torch.Tensor]:
        return self.active_buffer.filters_local

    def swap_buffers(self):
        """Activates the prefetched data (double_buffer_gpu.py:659-711)."""
        persistent_plan = self._persistent_plan
        if persistent_plan is not None:
            if self._before_persistent_apply is not None:
                self._before_persistent_apply()
            self._persistent_plan_layout(persistent_plan)
            source = self.loading_buffer
            target = self.active_buffer
            incoming_blocks = persistent_plan["incoming_blocks"]
            with torch.no_grad():
                self._copy_resident_blocks(source, target, incoming_blocks,
                                           persistent_plan["target_slices"])
            target.block_to_local_slice = dict(persistent_plan["next_slices"])
            target.loaded_blocks = list(persistent_plan["next_order"])
            target.resident_blocks = list(persistent_plan["keep_blocks"])
            target.streamed_blocks = list(incoming_blocks)
            target.evicted_blocks = list(persistent_plan["evicted_blocks"])
            target.num_gaussians = int(target.xyz.shape[0])
            target._block_starts = persistent_plan["block_starts"]
            # the slot copy above reads the staging buffer on this stream
            self._retire(source, torch.cuda.current_stream(self.device))
            source.clear()
            with self.lock:
                self._persistent_plan = None
                self._before_persistent_apply = None
                self.prefetch_in_progress = False
                self.stats["swaps"] += 1
                self.stats["persistent_slot_updates"] += 1
                self.stats["persistent_streamed_blocks"] += len(incoming_blocks)
            return
        with self.lock:
            if self.prefetch_in_progress:
                self.prefetch_complete_event.synchronize()
                if self.resident_refresh_complete_event is not None:
                    self.resident_refresh_complete_event.synchronize()
                self.prefetch_in_progress = False
            self.active_buffer_idx = 1 - self.active_buffer_idx
            self.stats["swaps"] += 1

    @staticmethod
    def _component_columns(layout) -> Dict[str, slice]:
        return component_columns(layout)

    def _allocate_target_tensors(self, target: GPUBuffer, num_rows: int) -> None:
        kw = dict(device=self.device, dtype=torch.float32)
        target.xyz = torch.empty(num_rows, 3, **kw)
        target.scaling = torch.empty(num_rows, 3, **kw)
        target.rotation = torch.empty(num_rows, 4, **kw)
        target.opacity = torch.empty(num_rows, 1, **kw)
        target.features_dc = torch.empty(num_rows, 3, **kw)
        target.features_rest = torch.empty(num_rows, 45, **kw)
        target.local_to_global_idx = torch.empty(num_rows, device=self.device, dtype=torch.long)

    def _acquire_host_staging(self, required_rows: int, host: bool = True
                              ) -> Tuple[Optional[torch.Tensor], torch.Tensor, int]:
        """Two rotating (pinned host, device) staging pairs; a slot is reused
        once its previous H2D has completed (double_buffer_gpu.py:748-809).
        host=False serves callers that DMA straight from page-locked blocks and
        need only the device half."""
        slot_idx = self._next_host_staging_slot
        self._next_host_staging_slot = (slot_idx + 1) % len(self._host_staging_slots)
        previous_copy = self._host_staging_events[slot_idx]
        if previous_copy is not None:
            previous_copy.synchronize()
        staging = self._host_staging_slots[slot_idx]
        gpu_staging = self._gpu_staging_slots[slot_idx]
        fits = required_rows <= self._host_staging_capacities[slot_idx]
        if fits and gpu_staging is not None and (staging is not None or not host):
            host_view = staging[:required_rows] if staging is not None else None
            return host_view, gpu_staging[:required_rows], slot_idx
        if not host:
            if not fits or gpu_staging is None:
                gpu_staging = torch.empty((required_rows, 59), dtype=torch.float32,
                                          device=self.device)
                self._gpu_staging_slots[slot_idx] = gpu_staging
                self._host_staging_slots[slot_idx] = None
                self._host_staging_capacities[slot_idx] = required_rows
            return None, gpu_staging[:required_rows], slot_idx
        try:
            staging = torch.empty((required_rows, 59), dtype=torch.float32, pin_memory=True)
        except RuntimeError:
            staging = torch.empty((required_rows, 59), dtype=torch.float32)
        gpu_staging = torch.empty((required_rows, 59), dtype=torch.float32, device=self.device)
        self._host_staging_slots[slot_idx] = staging
        self._gpu_staging_slots[slot_idx] = gpu_staging
        self._host_staging_capacities[slot_idx] = required_rows
        slots = [s for s in self._host_staging_slots if s is not None]
        self.stats["host_staging_bytes"] = sum(s.numel() * s.element_size() for s in slots)
        self.stats["host_staging_pinned"] = all(s.is_pinned() for s in slots)
        return staging[:required_rows], gpu_staging[:required_rows], slot_idx

    def _pack_streamed_blocks(self, block_ids, block_lengths, reader_blocks, reader_layout):
        total_rows = sum(block_lengths[b] for b in block_ids)
        staging, gpu_staging, slot_idx = self._acquire_host_staging(total_rows)
        output = staging[:total_rows]
        pieces = [reader_blocks[b][:block_lengths[b]] for b in block_ids]
        if len(pieces) == 1:
            output.copy_(pieces[0])
        else:
            torch.cat(pieces, dim=0, out=output)
        return output, gpu_staging[:total_rows], total_rows, slot_idx

    def _copy_resident_blocks(self, source: GPUBuffer, target: GPUBuffer, block_ids: List[int],
                              target_slices: Dict[int, slice]) -> int:
        """Block-granular slot remap source slice -> target slice for all six
        components and the global ids (double_buffer_gpu.py:811-872)."""
        if not block_ids:
            return 0
        src_starts = [int(source.block_to_local_slice[b].start) for b in block_ids]
        dst_starts = [int(target_slices[b].start) for b in block_ids]
        rows = [int(target_slices[b].stop - target_slices[b].start) for b in block_ids]
        return _ops.copy_blocks(source.components(), source.local_to_global_idx,
                                target.components(), target.local_to_global_idx,
                                src_starts, dst_starts, rows, self.device, err=self._err)

    def finalize_retained_blocks(self, block_ids: List[int], target: str = "loading"
                                 ) -> ResidentHandoffResult:
        persistent_plan = self._persistent_plan
        if target == "loading" and persistent_plan is not None:
            requested = set(int(b) for b in block_ids)
            reused = len(requested & persistent_plan["keep_set"])
            with self.lock:
                self._prefetch_finalized = True
                self._deferred_resident_blocks = []
                self.stats["persistent_omega_reuses"] += reused
            return ResidentHandoffResult(ready_blocks=reused, copied_blocks=0)

        if target == "loading":
            self._wait_for_target_layout()
        source_buffer = self.active_buffer
        target_buffer = self.loading_buffer if target == "loading" else self.active_buffer
        if source_buffer.is_empty() or target_buffer.is_empty() or not block_ids:
            return ResidentHandoffResult(ready_blocks=0, copied_blocks=0)
        refresh_ids = sorted(
            int(b) for b in set(block_ids)
            if int(b) in source_buffer.block_to_local_slice
            and int(b) in target_buffer.block_to_local_slice
        )
        if not refresh_ids:
            return ResidentHandoffResult(ready_blocks=0, copied_blocks=0)
        with torch.cuda.stream(self.resident_refresh_stream):
            self.resident_refresh_stream.wait_stream(torch.cuda.current_stream(self.device))
            self._copy_resident_blocks(source_buffer, target_buffer, refresh_ids,
                                       target_buffer.block_to_local_slice)
            resident_event = torch.cuda.Event()
            resident_event.record(self.resident_refresh_stream)
            self.resident_refresh_complete_event = resident_event
        with self.lock:
            self._prefetch_finalized = True
            self._deferred_resident_blocks = []
            self.stats["resident_refresh_blocks"] += len(refresh_ids)
        return ResidentHandoffResult(ready_blocks=len(refresh_ids), copied_blocks=len(refresh_ids))

    def _raise_if_prefetch_failed(self) -> None:
        """Re-raises, on the caller's thread, an error the N+1 worker died of."""
        job = self._prefetch_future
        if job is not None and job.done() and job.exception() is not None:
            raise job.exception()

    def _wait_for_target_layout(self) -> None:
        """Blocks until the N+1 worker has published the loading buffer's
        layout, polling for a failed worker every 10 ms."""
        ready = self._target_layout_ready
        while not ready.is_set():
            self._raise_if_prefetch_failed()
            ready.wait(timeout=0.01)
        self._raise_if_prefetch_failed()

    def _fill_streamed_global_ids(self, target: GPUBuffer, block_ids: List[int],
                                  target_offset: int, num_rows: int) -> None:
        if not block_ids:
            return
        ids = _ops.i64_to_device(block_ids, self.device)
        _ops.fill_global_ids(target.local_to_global_idx, target_offset, ids, num_rows,
                             self.block_size)

    # ------------------------------------------------------------------
    # Materialization (double_buffer_gpu.py:963-1105)
    # ------------------------------------------------------------------
    def _materialize_from_block_reader(self, target: GPUBuffer, source: GPUBuffer,
                                       sorted_visible_blocks: List[int], resident_set: set,
                                       evicted_set: set, allow_resident_copy: bool, block_reader,
                                       defer_resident_copy: bool = False) -> None:
        visible_set = set(sorted_visible_blocks)
        resident_blocks = sorted(
            b for b in visible_set & resident_set
            if allow_resident_copy and source is not None and not source.is_empty()
            and b in source.block_to_local_slice
        )
        streamed_blocks = sorted(visible_set - set(resident_blocks))
        target_order = resident_blocks + streamed_blocks
        block_lengths = {b: min(self.block_size, self.num_total - b * self.block_size)
                         for b in target_order}
        invalid = [b for b, n in block_lengths.items() if n <= 0]
        if invalid:
            raise ValueError(f"Invalid block IDs during N+1 materialization: {invalid}")
        offset = 0
        for b in target_order:
            target.block_to_local_slice[b] = slice(offset, offset + block_lengths[b])
            offset += block_lengths[b]
        self._allocate_target_tensors(target, offset)
        self._target_layout_ready.set()

        resident_rows = sum(block_lengths[b] for b in resident_blocks)
        if not defer_resident_copy:
            self._copy_resident_blocks(source, target, resident_blocks, target.block_to_local_slice)

        if streamed_blocks:
            streamed_rows = sum(block_lengths[b] for b in streamed_blocks)
            pointer_reader = getattr(block_reader, "block_host_pointers", None)
            pinned_reader = getattr(block_reader, "read_blocks_pinned", None)
            read_batch = getattr(block_reader, "read_batch", None)
            self._mark_prefetch("h2d_start")
            if callable(pointer_reader) or callable(pinned_reader):
                # Page-locked pool: one DMA per block straight into device
                # staging, no CPU-side concatenation.
                _, packed_gpu, staging_slot = self._acquire_host_staging(streamed_rows, host=False)
                want = np.asarray([block_lengths[b] for b in streamed_blocks], np.int64)
                if callable(pointer_reader):
                    src, rows = pointer_reader(streamed_blocks)
                    if np.any(rows < want):
                        raise ValueError("Invalid pinned blocks: fewer rows than the scene holds")
                else:
                    blocks = pinned_reader(streamed_blocks)
                    missing = [b for b in streamed_blocks if b not in blocks]
                    if missing:
                        raise KeyError(f"BlockReader omitted {len(missing)} N+1 blocks; "
                                       f"first missing={missing[:8]}")
                    for b in streamed_blocks:
                        host = blocks[b]
                        if host.shape[0] < block_lengths[b] or not host.is_contiguous():
                            raise ValueError(f"Invalid pinned block {b}: shape {tuple(host.shape)}")
                    src = np.asarray([blocks[b].data_ptr() for b in streamed_blocks], np.int64)
                nbytes = want * (59 * 4)
                row_off = np.concatenate([[0], np.cumsum(want)[:-1]]).astype(np.int64)
                dst = packed_gpu.data_ptr() + row_off * (59 * 4)
                ids_all = _ops.i64_to_device(streamed_blocks, self.device)
                # DMA in chunks on this stream; each chunk is unpacked on the
                # unpack stream as soon as its copies have landed, so only
                # the last chunk's unpack follows the DMA
                dma_stream = torch.cuda.current_stream(self.device)
                for c0 in range(0, len(streamed_blocks), self.PREFETCH_CHUNK_BLOCKS):
                    c1 = min(len(streamed_blocks), c0 + self.PREFETCH_CHUNK_BLOCKS)
                    _ops.h2d_blocks(dst[c0:c1].tolist(), src[c0:c1].tolist(),
                                    nbytes[c0:c1].tolist(), self.device)
                    landed = torch.cuda.Event()
                    landed.record(dma_stream)
                    self._unpack_stream.wait_event(landed)
                    r0 = int(row_off[c0])
                    r1 = int(row_off[c1 - 1] + want[c1 - 1])
                    with torch.cuda.stream(self._unpack_stream):
                        _ops.unpack_rows(packed_gpu[r0:r1], layout_code(block_reader.layout),
                                         target.components(), resident_rows + r0,
                                         global_ids=target.local_to_global_idx,
                                         block_ids=ids_all[c0:c1], block_size=self.block_size,
                                         err=self._err)
                self._mark_prefetch("h2d_end")
                note_reads = getattr(block_reader, "note_dma_reads", None)
                if callable(note_reads):
                    # the reader's entries are not rewritten before the DMAs ran
                    read_done = torch.cuda.Event()
                    read_done.record(dma_stream)
                    note_reads(streamed_blocks, read_done)
                dma_stream.wait_stream(self._unpack_stream)
                ids_all.record_stream(self._unpack_stream)
                packed_gpu.record_stream(self._unpack_stream)
                self.stats["direct_block_dma_calls"] += len(streamed_blocks)
                self._finish_streamed(target, staging_slot)
            else:
                if callable(read_batch):
                    staging, packed_gpu, staging_slot = self._acquire_host_staging(streamed_rows)
                    block_batch = read_batch(streamed_blocks, out=staging[:streamed_rows])
                    packed_cpu = block_batch.tensor
                    if tuple(packed_cpu.shape) != (streamed_rows, 59):
                        raise ValueError(
                            f"Invalid N+1 block batch shape {tuple(packed_cpu.shape)}; "
                            f"expected {(streamed_rows, 59)}")
                    for b in streamed_blocks:
                        sl = block_batch.block_slices.get(b)
                        expected = block_lengths[b]
                        if sl is None or sl.stop - sl.start != expected:
                            raise ValueError(
                                f"Invalid N+1 batch slice for block {b}: got={sl}, "
                                f"expected_rows={expected}")
                else:
                    reader_blocks = block_reader.read_blocks(streamed_blocks)
                    missing = [b for b in streamed_blocks if b not in reader_blocks]
                    if missing:
                        raise KeyError(
                            f"BlockReader omitted {len(missing)} N+1 blocks; first missing={missing[:8]}")
                    packed_cpu, packed_gpu, streamed_rows, staging_slot = self._pack_streamed_blocks(
                        streamed_blocks, block_lengths, reader_blocks, block_reader.layout)
                packed_gpu.copy_(packed_cpu, non_blocking=packed_cpu.is_pinned())
                self._mark_prefetch("h2d_end")
                ids = _ops.i64_to_device(streamed_blocks, self.device)
                _ops.unpack_rows(packed_gpu, layout_code(block_reader.layout), target.components(),
                                 resident_rows, global_ids=target.local_to_global_idx,
                                 block_ids=ids, block_size=self.block_size, err=self._err)
                self._finish_streamed(target, staging_slot)
        else:
            streamed_rows = 0

        target.loaded_blocks = target_order
        target.num_gaussians = resident_rows + streamed_rows
        target.resident_blocks = resident_blocks
        target.streamed_blocks = streamed_blocks
        target.evicted_blocks = sorted(evicted_set)
        target._block_starts = _build_block_starts(target.block_to_local_slice, self.num_blocks,
                                                   self.device)
        self.stats["batched_materializations"] += 1
        self.stats["batched_resident_blocks"] += len(resident_blocks)
        self.stats["batched_streamed_blocks"] += len(streamed_blocks)

    def _finish_streamed(self, target: GPUBuffer, staging_slot: int) -> None:
        """Streamed rows are unpacked (on the current stream): the staging
        slot may be reused once this point has been reached."""
        self._mark_prefetch("unpack_end")
        staging_event = torch.cuda.Event()
        staging_event.record(torch.cuda.current_stream(self.device))
        self._host_staging_events[staging_slot] = staging_event
        self.stats["batched_h2d_calls"] += 1

    def _local_filters(self, target: GPUBuffer, filters_global) -> List[torch.Tensor]:
        out = []
        for fg in filters_global:
            if fg is not None and len(fg) > 0:
                out.append(_ops.global_to_local_compact(fg.to(self.device), target._block_starts,
                                                        self.block_size))
            else:
                out.append(torch.empty(0, dtype=torch.long, device=self.device))
        return out

    def _run_block_reader_prefetch(self, *, target_buffer: GPUBuffer, source_buffer: GPUBuffer,
                                   sorted_visible_blocks: List[int], resident_set: set,
                                   evicted_set: set, filters_global: List[torch.Tensor],
                                   allow_resident_copy: bool, defer_resident_copy: bool,
                                   block_reader, before_target_reuse, caller_stream=None) -> None:
        start_time = time.time()
        if before_target_reuse is not None:
            before_target_reuse()
        with torch.cuda.device(self.device), torch.cuda.stream(self.prefetch_stream):
            # the buffer being refilled was last used by the caller's stream
            # (optimizer, slot copies) and the resident-refresh stream
            self._retire(target_buffer, *[st for st in (caller_stream, self.resident_refresh_stream)
                                          if st is not None])
            target_buffer.clear()
            if not sorted_visible_blocks:
                target_buffer.evicted_blocks = sorted(evicted_set)
                self._target_layout_ready.set()
                self.prefetch_complete_event.record(self.prefetch_stream)
                with self.lock:
                    self._prefetch_finalized = True
                return
            with torch.cuda.nvtx.range("Tide N+1: block read and pack"):
                self._materialize_from_block_reader(
                    target=target_buffer, source=source_buffer,
                    sorted_visible_blocks=sorted_visible_blocks, resident_set=resident_set,
                    evicted_set=evicted_set, allow_resident_copy=allow_resident_copy,
                    block_reader=block_reader, defer_resident_copy=defer_resident_copy)
            target_buffer.filters_local = self._local_filters(target_buffer, filters_global)
            deferred = target_buffer.resident_blocks if defer_resident_copy else []
            with self.lock:
                self._deferred_resident_blocks = list(deferred)
            self.prefetch_complete_event.record(self.prefetch_stream)
            if not deferred:
                with self.lock:
                    self._prefetch_finalized = True
        self.stats["total_prefetch_time_ms"] += (time.time() - start_time) * 1000.0

    #: blocks per DMA chunk of a page-locked prefetch (each chunk is unpacked
    #: while the next one is in flight)
    PREFETCH_CHUNK_BLOCKS = 128

    def _retire(self, buffer: GPUBuffer, *streams) -> None:
        """Keeps `buffer`'s device memory from being handed out again until
        the work already enqueued on `streams` (which read or wrote it) has
        run: the caching allocator would otherwise reuse it at once for the
        next allocation on the stream it was allocated on."""
        for t in (buffer.xyz, buffer.scaling, buffer.rotation, buffer.opacity,
                  buffer.features_dc, buffer.features_rest, buffer.local_to_global_idx,
                  buffer._block_starts):
            if t is not None:
                for st in streams:
                    t.record_stream(st)

    #: profiling hook (off by default): a dict that receives CUDA events
    #: recorded on the prefetch stream at "h2d_start", "h2d_end", "unpack_end"
    prefetch_events = None

    def _mark_prefetch(self, name: str) -> None:
        if self.prefetch_events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.prefetch_events[name] = ev

    def _open_prefetch(self, iteration: int) -> None:
        """Retires a prefetch still in flight (waiting for it), then resets
        the per-prefetch state for `iteration`."""
        with self.lock:
            running = self.prefetch_iteration if self.prefetch_in_progress else None
        if running is not None:
            self.wait_for_prefetch(running)
        fresh = {
            "prefetch_in_progress": True, "prefetch_iteration": iteration,
            "prefetch_complete_event": torch.cuda.Event(),
            "resident_refresh_complete_event": None, "_prefetch_finalized": False,
            "_deferred_resident_blocks": [], "_persistent_plan": None,
            "_before_persistent_apply": None,
        }
        with self.lock:
            for name, value in fresh.items():
                setattr(self, name, value)
            self._target_layout_ready.clear()

    def start_prefetch(self, iteration: int, visible_block_ids: List[int],
                       filters_global: Optional[List[torch.Tensor]] = None,
                       ram_cache: Optional[Dict[str, torch.Tensor]] = None,
                       unified_params: Optional[torch.Tensor] = None,
                       block_cache: Optional[Dict[int, torch.Tensor]] = None,
                       resident_block_ids: Optional[List[int]] = None,
                       evicted_block_ids: Optional[List[int]] = None,
                       allow_resident_copy: bool = True, block_reader: "Optional[object]" = None,
                       defer_resident_copy: bool = False, before_target_reuse=None):
        """Starts the N+1 prefetch into the loading buffer; returns at once for
        block readers (double_buffer_gpu.py:1169-1454)."""
        self._open_prefetch(iteration)

        if block_reader is not None:
            sorted_visible = sorted(set(map(int, visible_block_ids)))
            resident_set = set(map(int, resident_block_ids or []))
            evicted_set = set(map(int, evicted_block_ids or []))
            plan = self._build_persistent_plan(sorted_visible, resident_set, evicted_set,
                                               allow_resident_copy=allow_resident_copy,
                                               defer_resident_copy=defer_resident_copy)
            if plan is not None:
                self._persistent_plan = plan
                self._before_persistent_apply = before_target_reuse
                prefetch_blocks = plan["incoming_blocks"]
                prefetch_resident_set = set()
                prefetch_deferred = False
                worker_fence = None
            else:
                self.stats["persistent_ab_fallbacks"] += 1
                prefetch_blocks = sorted_visible
                prefetch_resident_set = resident_set
                prefetch_deferred = defer_resident_copy
                worker_fence = before_target_reuse
            job = dict(
                target_buffer=self.loading_buffer, source_buffer=self.active_buffer,
                sorted_visible_blocks=prefetch_blocks, resident_set=prefetch_resident_set,
                evicted_set=evicted_set, filters_global=list(filters_global or []),
                allow_resident_copy=allow_resident_copy, defer_resident_copy=prefetch_deferred,
                block_reader=block_reader, before_target_reuse=worker_fence,
                caller_stream=torch.cuda.current_stream(self.device))
            if (plan is not None and worker_fence is None
                    and callable(getattr(block_reader, "block_host_pointers", None))):
                # A page-locked pool: reading is a pointer lookup, so the whole
                # materialization only enqueues GPU work (DMA + unpack). Doing
                # it here starts the DMA at once instead of when the worker
                # thread next gets the interpreter lock.
                future = Future()
                try:
                    self._run_block_reader_prefetch(**job)
                    # the slot map of the next step, built while the DMA runs
                    self._persistent_plan_layout(plan)
                    future.set_result(None)
                except BaseException as exc:  # surfaced by wait_for_prefetch
                    future.set_exception(exc)
                self._prefetch_future = future
                self._target_layout_ready.set()
                self.stats["inline_prefetches"] += 1
                return
            self._prefetch_future = self._prefetch_executor.submit(
                self._run_block_reader_prefetch, **job)
            self._prefetch_future.add_done_callback(lambda _f: self._target_layout_ready.set())
            return
        self._legacy_prefetch(visible_block_ids, filters_global, ram_cache, unified_params,
                              block_cache, resident_block_ids, evicted_block_ids,
                              allow_resident_copy)

    def _legacy_prefetch(self, visible_block_ids, filters_global, ram_cache, unified_params,
                         block_cache, resident_block_ids, evicted_block_ids,
                         allow_resident_copy) -> None:
        """Synchronous-source prefetch (no block reader): blocks in ascending
        order, retained blocks copied from the active buffer, the rest taken
        from unified_params / block_cache / ram_cache
        (double_buffer_gpu.py:1277-1454)."""
        caller_stream = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device), torch.cuda.stream(self.prefetch_stream):
            start_time = time.time()
            target = self.loading_buffer
            source = self.active_buffer
            self._retire(target, caller_stream, self.resident_refresh_stream)
            target.clear()
            sorted_visible = sorted(set(int(b) for b in visible_block_ids))
            resident_set = set(int(b) for b in (resident_block_ids or []))
            evicted_set = set(int(b) for b in (evicted_block_ids or []))
            filters_global = filters_global or []
            if not sorted_visible:
                target.evicted_blocks = sorted(evicted_set)
                self._target_layout_ready.set()
                self.prefetch_complete_event.record(self.prefetch_stream)
                return
            lengths = {b: min(b * self.block_size + self.block_size, self.num_total)
                       - b * self.block_size for b in sorted_visible}
            num_visible = sum(lengths.values())
            self._allocate_target_tensors(target, num_visible)
            copy_plan = ([], [], [])
            stream_plan = []
            resident_used, streamed_used = [], []
            offset = 0
            for b in sorted_visible:
                n = lengths[b]
                target.block_to_local_slice[b] = slice(offset, offset + n)
                start_idx = b * self.block_size
                can_copy = (allow_resident_copy and b in resident_set and source is not None
                            and source.block_to_local_slice is not None
                            and b in source.block_to_local_slice and not source.is_empty())
                if can_copy:
                    copy_plan[0].append(int(source.block_to_local_slice[b].start))
                    copy_plan[1].append(offset)
                    copy_plan[2].append(n)
                    resident_used.append(b)
                elif unified_params is not None:
                    stream_plan.append((offset, unified_params[start_idx:start_idx + n], "unified"))
                    streamed_used.append(b)
                elif block_cache is not None:
                    if b not in block_cache:
                        raise KeyError(f"Block {b} missing from block_cache during double-buffer prefetch")
                    stream_plan.append((offset, block_cache[b][:n], "cache"))
                    streamed_used.append(b)
                else:
                    if ram_cache is None:
                        raise ValueError("Either block_reader, unified_params, block_cache, or "
                                         "ram_cache must be provided")
                    ids = torch.arange(start_idx, start_idx + n, dtype=torch.long)
                    packed = torch.empty((n, 59), dtype=torch.float32)
                    cols = component_columns("cache")
                    for name in ("xyz", "scaling", "rotation", "opacity"):
                        packed[:, cols[name]] = ram_cache[name][ids]
                    if "features_dc" in ram_cache:
                        packed[:, 11:14] = ram_cache["features_dc"][ids]
                        packed[:, 14:59] = ram_cache["features_rest"][ids]
                    elif "sh_cache" in ram_cache:
                        sh = ram_cache["sh_cache"][ids]
                        packed[:, 11:14] = sh[:, :3]
                        packed[:, 14:59] = sh[:, 3:48]
                    else:
                        raise KeyError("ram_cache must contain either features_dc/features_rest or sh_cache")
                    stream_plan.append((offset, packed, "cache"))
                    streamed_used.append(b)
                offset += n
            if copy_plan[2]:
                _ops.copy_blocks(source.components(), None, target.components(), None,
                                 copy_plan[0], copy_plan[1], copy_plan[2], self.device)
            for dst_off, host, layout in stream_plan:
                packed_gpu = host.contiguous().to(self.device, non_blocking=host.is_pinned())
                _ops.unpack_rows(packed_gpu, layout_code(layout), target.components(), dst_off)
            ids_dev = _ops.i64_to_device(sorted_visible, self.device)
            _ops.fill_global_ids(target.local_to_global_idx, 0, ids_dev, num_visible,
                                 self.block_size)
            target.loaded_blocks = sorted_visible
            target.num_gaussians = num_visible
            target.resident_blocks = resident_used
            target.streamed_blocks = streamed_used
            target.evicted_blocks = sorted(evicted_set)
            target._block_starts = _build_block_starts(target.block_to_local_slice,
                                                       self.num_blocks, self.device)
            self._target_layout_ready.set()
            target.filters_local = self._local_filters(target, filters_global)
            self.prefetch_complete_event.record(self.prefetch_stream)
            self.stats["total_prefetch_time_ms"] += (time.time() - start_time) * 1000

    def refresh_blocks_from_block_cache(self, block_cache: Dict[int, torch.Tensor],
                                        block_ids: List[int], target: str = "loading") -> int:
        """Overwrites retained blocks from CACHE-layout host tensors
        (double_buffer_gpu.py:1455-1506)."""
        target_buffer = self.loading_buffer if target == "loading" else self.active_buffer
        if target_buffer.is_empty() or not block_ids:
            return 0
        refreshed = 0
        with torch.cuda.stream(self.prefetch_stream):
            for b in block_ids:
                if b not in target_buffer.block_to_local_slice or b not in block_cache:
                    continue
                sl = target_buffer.block_to_local_slice[b]
                block_len = sl.stop - sl.start
                tensor = block_cache[b]
                if block_len <= 0 or tensor is None or tensor.numel() == 0:
                    continue
                n = min(block_len, int(tensor.shape[0]))
                if n <= 0:
                    continue
                packed_gpu = tensor[:n].contiguous().to(self.device, non_blocking=tensor.is_pinned())
                _ops.unpack_rows(packed_gpu, _lib.LAYOUT_CACHE, target_buffer.components(), sl.start)
                refreshed += 1
            if refreshed > 0:
                self.prefetch_complete_event.record(self.prefetch_stream)
        return refreshed

    def wait_for_prefetch(self, iteration: int) -> bool:
        with self.lock:
            if not self.prefetch_in_progress or self.prefetch_iteration != iteration:
                self.stats["prefetch_misses"] += 1
                return False
        prefetch_future = self._prefetch_future
        if prefetch_future is not None:
            prefetch_future.result()
        with self.lock:
            finalized = self._prefetch_finalized
            deferred = list(self._deferred_resident_blocks)
        if not finalized:
            handoff = self.finalize_retained_blocks(deferred, target="loading")
            if handoff.ready_blocks != len(deferred):
                raise RuntimeError(
                    "N+1 retained-block handoff was incomplete: "
                    f"expected={len(deferred)} ready={handoff.ready_blocks}")
        resident_event = self.resident_refresh_complete_event
        if not (self.prefetch_complete_event.query()
                and (resident_event is None or resident_event.query())):
            self.prefetch_complete_event.synchronize()
            if resident_event is not None:
                resident_event.synchronize()
        self._check_device_errors()
        self.stats["prefetch_hits"] += 1
        with self.lock:
            self.prefetch_in_progress = False
        return True

    def _check_device_errors(self) -> None:
        problem = _lib.decode_device_error(self._err.cpu().tolist())
        if problem is not None:
            self._err.zero_()
            raise RuntimeError(f"[DoubleBufferGPU] device copy failed: {problem}")

    def load_visible_blocks_sync(self, visible_block_ids: List[int],
                                 filters_global: List[torch.Tensor],
                                 unified_params: torch.Tensor) -> Dict[str, torch.Tensor]:
        """Synchronous load into the active buffer (double_buffer_gpu.py:1567-1645)."""
        target = self.active_buffer
        self._retire(target, self.prefetch_stream, self.resident_refresh_stream)
        target.clear()
        if len(visible_block_ids) == 0:
            raise ValueError("No visible blocks to load!")
        ordered = sorted(visible_block_ids)
        ids = np.concatenate([np.arange(b * self.block_size,
                                        min(b * self.block_size + self.block_size, self.num_total))
                              for b in ordered]).astype(np.int64)
        idx = torch.from_numpy(ids)
        packed = unified_params[idx].contiguous()
        self._allocate_target_tensors(target, int(ids.size))
        packed_gpu = packed.to(self.device)
        _ops.unpack_rows(packed_gpu, _lib.LAYOUT_UNIFIED, target.components(), 0)
        target.local_to_global_idx = idx.to(self.device)
        target.loaded_blocks = sorted(visible_block_ids)
        target.num_gaussians = int(ids.size)
        block_to_slice: Dict[int, slice] = {}
        offset = 0
        for b in ordered:
            n = min(b * self.block_size + self.block_size, self.num_total) - b * self.block_size
            block_to_slice[b] = slice(offset, offset + n)
            offset += n
        target.block_to_local_slice = block_to_slice
        target._block_starts = _build_block_starts(block_to_slice, self.num_blocks, self.device)
        target.filters_local = self._local_filters(target, filters_global)
        return {"xyz": target.xyz, "scaling": target.scaling, "rotation": target.rotation,
                "opacity": target.opacity, "features_dc": target.features_dc,
                "features_rest": target.features_rest}

    def update_ram_cache(self, geometry_cache: Optional[Dict[str, torch.Tensor]] = None,
                         sh_cache: Optional[torch.Tensor] = None,
                         unified_params: Optional[torch.Tensor] = None):
        """Active buffer -> host tables by global id (double_buffer_gpu.py:1647-1686)."""
        buf = self.active_buffer
        if buf.is_empty():
            return
        rows = int(buf.xyz.shape[0])
        layout = _lib.LAYOUT_UNIFIED if unified_params is not None else _lib.LAYOUT_CACHE
        packed = torch.empty((rows, 59), dtype=torch.float32, device=self.device)
        _ops.pack_rows(buf.components(), [0], [rows], packed, layout)
        host = packed.cpu()
        global_ids = buf.local_to_global_idx.cpu()
        if unified_params is not None:
            unified_params[global_ids] = host
            return
        cols = component_columns("cache")
        if geometry_cache is not None:
            for name in ("xyz", "scaling", "rotation", "opacity"):
                geometry_cache[name][global_ids] = host[:, cols[name]]
        if sh_cache is not None:
            sh_cache[global_ids] = host[:, 11:59]

    def get_stats(self) -> Dict[str, object]:
        stats = self.stats.copy()
        total = stats["prefetch_hits"] + stats["prefetch_misses"]
        stats["hit_rate"] = stats["prefetch_hits"] / total if total > 0 else 0.0
        stats["avg_prefetch_time_ms"] = (stats["total_prefetch_time_ms"] / stats["prefetch_hits"]
                                         if stats["prefetch_hits"] > 0 else 0.0)
        stats["active_buffer"] = "A" if self.active_buffer_idx == 0 else "B"
        stats["active_gaussians"] = self.active_buffer.num_gaussians
        stats["active_blocks"] = len(self.active_buffer.loaded_blocks)
        return stats

    def _reset_host_staging(self) -> None:
        """Drops the two rotating host/device staging slots."""
        self._host_staging_slots = [None] * 2
        self._gpu_staging_slots = [None] * 2
        self._host_staging_capacities = [0] * 2
        self._host_staging_events = [None] * 2
        self.stats.update(host_staging_bytes=0, host_staging_pinned=False)

    def clear(self):
        """Finishes the worker jobs and both streams, stops the workers, then
        releases the buffers and staging slots and forgets every dirty mark
        (the reference's clear, double_buffer_gpu.py:1711-1731)."""
        for job in (self._resident_plan_future, self._prefetch_future):
            if job is not None:
                job.result()
        for stream in (self.prefetch_stream, self.resident_refresh_stream):
            stream.synchronize()
        if not self._executor_shutdown:
            for pool in (self._prefetch_executor, self._resident_plan_executor):
                pool.shutdown(wait=True)
            self._executor_shutdown = True
        for buf in (self.buffer_a, self.buffer_b):
            buf.clear()
        self._reset_host_staging()
        self._target_layout_ready.clear()
        self.resident_refresh_complete_event = None
        self._dirty_bitmap.zero_()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()

    def __del__(self):
        try:
            self.clear()
        except Exception:
            pass


def get_next_iteration_blocks(storage_adapter, training_schedule: List[int], iteration: int,
                              batch_size: int, schedule_ordering: str = "trajectory"
                              ) -> Tuple[List[int], List[int]]:
    """Visible blocks of the next scheduled batch (double_buffer_gpu.py:746-777)."""
    from storage.schedule_utils import get_current_and_next_camera_batches

    _, next_batch = get_current_and_next_camera_batches(
        training_schedule=training_schedule, iteration=iteration, batch_size=batch_size,
        schedule_ordering=schedule_ordering)
    visible = set()
    for cam_id in next_batch.batch_indices:
        visible.update(storage_adapter.get_visible_blocks(cam_id))
    return next_batch.batch_indices, sorted(visible)
