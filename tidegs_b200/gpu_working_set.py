"""GPU working set and the write-back gather (drop-in for TideGS's
strategies/tide_engine/gpu_working_set.py: PendingBlockBounds :118-129,
PendingBlockWriteback :132-184, GPUWorkingSet :187-1119).

Device work goes through libtidegs_b200.so:
* stage_updated_blocks (:895-988): SoA -> packed CACHE rows in one launch of
  `tgs_pack_rows` (component ranges staged in shared memory by bulk copies), then
  one D2H into rotating pinned staging on the write-back stream.
* stage_block_bounds (:990-1061): `tgs_block_bounds`, exact min/max per block.
* load_visible_blocks_with_retention (:447-793): retained blocks move with the
  slot-remap copy kernel, cold blocks arrive as packed rows (one H2D) and are
  scattered into the component arrays by `tgs_unpack_rows`.
* global_to_local (:312-333): `tgs_global_to_local`.
"""
from __future__ import annotations

import os
import threading
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib, _ops
from .block_reader import component_columns, layout_code

COMPONENT_NAMES = ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest")
_WIDTHS = _ops.WIDTHS


def _pinned_empty(shape, dtype=torch.float32) -> torch.Tensor:
    try:
        return torch.empty(shape, dtype=dtype, pin_memory=True)
    except RuntimeError:
        return torch.empty(shape, dtype=dtype)


class PendingBlockBounds:
    """Compact per-block bounds awaiting one asynchronous D2H copy."""

    def __init__(self, block_ids, cpu_bounds, ready_event, gpu_bounds=None):
        self.block_ids = list(block_ids)
        self.cpu_bounds = cpu_bounds
        self.ready_event = ready_event
        self.gpu_bounds = gpu_bounds

    def wait(self) -> Tuple[List[int], torch.Tensor]:
        self.ready_event.synchronize()
        return self.block_ids, self.cpu_bounds


class PendingBlockWriteback:
    """One batched GPU-to-CPU writeback awaiting a single CUDA event."""

    COMPONENT_ORDER = COMPONENT_NAMES

    def __init__(self, plans, packed_cpu, ready_event, release_event=None, gpu_refs=None):
        self.plans = plans
        self.packed_cpu = packed_cpu
        self.ready_event = ready_event
        self.release_event = release_event
        self.gpu_refs = list(gpu_refs or [])
        self._result = None
        self._wait_lock = threading.Lock()

    @property
    def block_ids(self) -> List[int]:
        return [int(block_id) for block_id, _ in self.plans]

    def wait_gpu(self) -> None:
        self.ready_event.synchronize()

    def wait(self) -> Dict[int, torch.Tensor]:
        if self._result is not None:
            return self._result
        with self._wait_lock:
            if self._result is not None:
                return self._result
            self.wait_gpu()
            result: Dict[int, torch.Tensor] = {}
            offset = 0
            for block_id, row_count in self.plans:
                result[block_id] = self.packed_cpu[offset:offset + row_count]
                offset += row_count
            self._result = result
        return result

    def release(self) -> None:
        if self.release_event is not None:
            self.release_event.set()


class PendingCacheWriteback(PendingBlockWriteback):
    """A write-back whose per-block DMAs land in fresh entries of a host block
    cache: `wait()` publishes them there (each block dirty, version + 1) and
    returns {block: entry view}. There is no staging copy, so `packed_cpu`
    is None."""

    def __init__(self, plans, ready_event, host_cache, views, gpu_refs=None):
        super().__init__(plans, None, ready_event, gpu_refs=gpu_refs)
        self.host_cache = host_cache
        self._views = list(views)

    def wait(self) -> Dict[int, torch.Tensor]:
        if self._result is not None:
            return self._result
        with self._wait_lock:
            if self._result is None:
                self.wait_gpu()
                self.host_cache.commit_writeback(self.plans, self._views)
                self._result = {b: v for (b, _), v in zip(self.plans, self._views)}
        return self._result

    def release(self) -> None:
        self.wait()


class GPUWorkingSet:
    """GPU working set of the resident blocks (59 fp32 columns per Gaussian,
    stored as six contiguous component tensors)."""

    def __init__(self, num_total_gaussians: int, block_size: int, device: str = "cuda",
                 verbose: bool = False):
        self.num_total = int(num_total_gaussians)
        self.block_size = int(block_size)
        self.device = _lib.require_cuda(device, "GPUWorkingSet")
        self.num_blocks = (self.num_total + self.block_size - 1) // self.block_size
        self.verbose = bool(verbose)

        self.gpu_xyz: Optional[torch.Tensor] = None
        self.gpu_scaling: Optional[torch.Tensor] = None
        self.gpu_rotation: Optional[torch.Tensor] = None
        self.gpu_opacity: Optional[torch.Tensor] = None
        self.gpu_features_dc: Optional[torch.Tensor] = None
        self.gpu_features_rest: Optional[torch.Tensor] = None

        self.previous_blocks: List[int] = []
        self.previous_block_data: Dict[int, Dict[str, torch.Tensor]] = {}
        self.hotspot_stats = {
            "total_iterations": 0,
            "total_blocks_loaded": 0,
            "total_blocks_retained": 0,
            "total_blocks_cold": 0,
        }
        self.block_to_gpu_slice: Dict[int, slice] = {}
        self.loaded_blocks: List[int] = []
        self.local_to_global_idx: Optional[torch.Tensor] = None
        self._block_starts: Optional[torch.Tensor] = None

        self._writeback_stream = torch.cuda.Stream(device=self.device)
        self._writeback_staging_slots: List[Optional[torch.Tensor]] = [None, None]
        self._writeback_gpu_staging_slots: List[Optional[torch.Tensor]] = [None, None]
        self._writeback_staging_capacities = [0, 0]
        self._writeback_slot_available = [threading.Event(), threading.Event()]
        for available in self._writeback_slot_available:
            available.set()
        self._next_writeback_slot = 0
        self.writeback_stats = {
            "batched_writebacks": 0,
            "batched_writeback_blocks": 0,
            "batched_writeback_rows": 0,
            "async_d2h_calls": 0,
            "pinned_staging_bytes": 0,
            "pinned_staging": False,
            "bounds_updates": 0,
            "direct_cache_d2h_blocks": 0,
        }
        self._direct_staging: Optional[torch.Tensor] = None
        self._log(f"[GPUWorkingSet] Initialized for {self.num_total:,} Gaussians")

    def _log(self, message: str) -> None:
        if self.verbose:
            print(message)

    # ------------------------------------------------------------------
    def _components(self) -> Dict[str, Optional[torch.Tensor]]:
        return {
            "xyz": self.gpu_xyz, "opacity": self.gpu_opacity, "scaling": self.gpu_scaling,
            "rotation": self.gpu_rotation, "features_dc": self.gpu_features_dc,
            "features_rest": self.gpu_features_rest,
        }

    def refresh_topology(self, num_total_gaussians: int):
        num_total_gaussians = int(num_total_gaussians)
        if num_total_gaussians == self.num_total:
            return
        self.num_total = num_total_gaussians
        self.num_blocks = (self.num_total + self.block_size - 1) // self.block_size
        self.clear()
        self.previous_blocks.clear()
        self.previous_block_data.clear()

    def _rebuild_block_starts(self) -> None:
        self._block_starts = _ops.build_block_starts(
            ((b, s.start) for b, s in self.block_to_gpu_slice.items()), self.num_blocks,
            self.device)

    def global_to_local(self, global_ids: torch.Tensor) -> torch.Tensor:
        if self._block_starts is None:
            self._rebuild_block_starts()
        return _ops.global_to_local(global_ids, self._block_starts, self.block_size)

    def _block_len(self, block_id: int) -> int:
        start = block_id * self.block_size
        return min(start + self.block_size, self.num_total) - start

    def _alloc_components(self, rows: int) -> Dict[str, torch.Tensor]:
        return {name: torch.empty(rows, _WIDTHS[name], device=self.device, dtype=torch.float32)
                for name in _ops.COMPONENTS}

    def _set_components(self, comps: Dict[str, torch.Tensor]) -> None:
        self.gpu_xyz = comps["xyz"]
        self.gpu_scaling = comps["scaling"]
        self.gpu_rotation = comps["rotation"]
        self.gpu_opacity = comps["opacity"]
        self.gpu_features_dc = comps["features_dc"]
        self.gpu_features_rest = comps["features_rest"]

    def _result_dict(self) -> Dict[str, torch.Tensor]:
        return {
            "xyz": self.gpu_xyz, "scaling": self.gpu_scaling, "rotation": self.gpu_rotation,
            "opacity": self.gpu_opacity, "features_dc": self.gpu_features_dc,
            "features_rest": self.gpu_features_rest,
        }

    def _upload_packed(self, packed_cpu: torch.Tensor, layout, comps: Dict[str, torch.Tensor],
                       target_offset: int) -> None:
        packed_gpu = packed_cpu.to(self.device, non_blocking=packed_cpu.is_pinned())
        _ops.unpack_rows(packed_gpu, layout_code(layout), comps, target_offset)

    def load_visible_blocks(self, visible_block_ids: List[int],
                            geometry_cache: Dict[str, torch.Tensor],
                            sh_cache: torch.Tensor) -> Dict[str, torch.Tensor]:
        """RAM caches (separate geometry tensors + (N,48) SH) -> working set
        (gpu_working_set.py:335-445)."""
        if len(visible_block_ids) == 0:
            raise ValueError("No visible blocks to load!")
        inferred = min(int(geometry_cache["xyz"].shape[0]), int(geometry_cache["scaling"].shape[0]),
                       int(geometry_cache["rotation"].shape[0]),
                       int(geometry_cache["opacity"].shape[0]), int(sh_cache.shape[0]))
        self.refresh_topology(inferred)
        self.clear()
        ordered = sorted(visible_block_ids)
        ids = np.concatenate([np.arange(b * self.block_size, min((b + 1) * self.block_size,
                                                                 self.num_total))
                              for b in ordered]).astype(np.int64)
        idx = torch.from_numpy(ids)
        packed = _pinned_empty((ids.size, 59))
        cols = component_columns("cache")
        packed[:, cols["xyz"]] = geometry_cache["xyz"][idx]
        packed[:, cols["scaling"]] = geometry_cache["scaling"][idx]
        packed[:, cols["rotation"]] = geometry_cache["rotation"][idx]
        packed[:, cols["opacity"]] = geometry_cache["opacity"][idx]
        sh = sh_cache[idx]
        packed[:, 11:14] = sh[:, :3]
        packed[:, 14:59] = sh[:, 3:48]
        comps = self._alloc_components(ids.size)
        self._upload_packed(packed, "cache", comps, 0)
        self._set_components(comps)
        self.loaded_blocks = sorted(set(int(b) for b in visible_block_ids
                                        if 0 <= int(b) < self.num_blocks))
        self.local_to_global_idx = idx.to(self.device)
        offset = 0
        for block_id in self.loaded_blocks:
            n = self._block_len(block_id)
            self.block_to_gpu_slice[block_id] = slice(offset, offset + n)
            offset += n
        return self._result_dict()

    def load_visible_blocks_with_retention(
        self,
        visible_block_ids: List[int],
        active_blocks_ram: Optional[Dict[int, torch.Tensor]] = None,
        enable_retention: bool = True,
        unified_params: "torch.Tensor | None" = None,
        block_reader: "Optional[object]" = None,
    ) -> Tuple[Dict[str, torch.Tensor], Dict[str, int]]:
        """Synchronous materialization with resident-overlap reuse
        (gpu_working_set.py:447-793)."""
        if block_reader is not None:
            self.refresh_topology(int(block_reader.total_gaussians))
        elif unified_params is not None:
            self.refresh_topology(int(unified_params.shape[0]))

        visible_set = set(int(b) for b in visible_block_ids if 0 <= int(b) < self.num_blocks)
        previous_set = set(self.previous_blocks)

        if len(visible_block_ids) == 0:
            print("[GPUWorkingSet WARNING] visible_block_ids is empty! Returning empty working set.")
            self._set_components(self._alloc_components(0))
            self.loaded_blocks = []
            self.local_to_global_idx = torch.empty(0, dtype=torch.long, device=self.device)
            self.previous_blocks = []
            self.block_to_gpu_slice.clear()
            stats = {"hotspot_count": 0, "cold_count": 0, "total_count": 0, "hit_rate": 0.0,
                     "memory_mb": 0.0, "num_gaussians": 0}
            return self._result_dict(), stats

        if enable_retention and len(previous_set) > 0:
            hotspot_blocks = list(visible_set & previous_set)
            cold_blocks = list(visible_set - previous_set)
        else:
            hotspot_blocks = []
            cold_blocks = list(visible_set)
        hotspot_count = len(hotspot_blocks)
        cold_count = len(cold_blocks)
        total_count = len(visible_block_ids)
        hit_rate = hotspot_count / total_count if total_count > 0 else 0.0
        self.hotspot_stats["total_iterations"] += 1
        self.hotspot_stats["total_blocks_loaded"] += total_count
        self.hotspot_stats["total_blocks_retained"] += hotspot_count
        self.hotspot_stats["total_blocks_cold"] += cold_count

        ssd_mode = (block_reader is not None) or (unified_params is not None)
        can_use_gpu_hotspots = (not ssd_mode and hotspot_count > 0 and self.gpu_xyz is not None)
        old_slices = dict(self.block_to_gpu_slice) if can_use_gpu_hotspots else {}
        old_comps = self._components() if can_use_gpu_hotspots else {}
        self.block_to_gpu_slice.clear()

        sorted_visible = sorted(visible_block_ids)
        lengths = [self._block_len(int(b)) for b in sorted_visible]
        total_rows = int(sum(lengths))
        comps = self._alloc_components(total_rows)

        cold_source: Optional[Dict[int, torch.Tensor]] = None
        cold_layout = None
        if block_reader is not None:
            cold_layout = block_reader.layout
            cold_ids = [b for b in sorted_visible if not (can_use_gpu_hotspots and b in old_slices)]
            cold_source = block_reader.read_blocks(cold_ids)

        reuse = ([], [], [])       # src starts, dst starts, rows (retained on GPU)
        stream_plan = []           # (dst_start, rows, host tensor, layout)
        zero_slices = []
        offset = 0
        for block_id, block_len in zip(sorted_visible, lengths):
            s = slice(offset, offset + block_len)
            if can_use_gpu_hotspots and block_id in old_slices:
                reuse[0].append(old_slices[block_id].start)
                reuse[1].append(offset)
                reuse[2].append(block_len)
            elif cold_source is not None and block_id in cold_source:
                stream_plan.append((offset, block_len, cold_source[block_id][:block_len], cold_layout))
            elif unified_params is not None:
                start_idx = block_id * self.block_size
                stream_plan.append((offset, block_len,
                                    unified_params.data[start_idx:start_idx + block_len], "unified"))
            elif active_blocks_ram is not None and block_id in active_blocks_ram:
                stream_plan.append((offset, block_len, active_blocks_ram[block_id][:block_len],
                                    "cache"))
            else:
                zero_slices.append(s)
                print(f"[WARNING] Block {block_id} not reachable via any source "
                      "(reader/unified_params/active_blocks_ram)")
            self.block_to_gpu_slice[block_id] = s
            offset += block_len

        if reuse[2]:
            _ops.copy_blocks(old_comps, None, comps, None, reuse[0], reuse[1], reuse[2],
                             self.device)
        self._stream_packed(stream_plan, comps)
        for s in zero_slices:
            for t in comps.values():
                t[s].zero_()
        if os.environ.get("FLEX3DGS_SYNC_DMA", "0") == "1":
            torch.cuda.synchronize()

        self._set_components(comps)
        self.loaded_blocks = sorted_visible
        gids = torch.empty(total_rows, dtype=torch.long, device=self.device)
        if total_rows:
            block_ids_dev = _ops.i64_to_device(sorted_visible, self.device)
            _ops.fill_global_ids(gids, 0, block_ids_dev, total_rows, self.block_size)
        self.local_to_global_idx = gids
        self._rebuild_block_starts()
        self.previous_blocks = sorted_visible.copy()

        memory_mb = total_rows * 59 * 4 / (1024 ** 2)
        stats = {
            "hotspot_count": hotspot_count,
            "cold_count": cold_count,
            "total_count": total_count,
            "hit_rate": hit_rate,
            "memory_mb": memory_mb,
            "num_gaussians": total_rows,
            "data_reused_count": hotspot_count if can_use_gpu_hotspots else 0,
        }
        return self._result_dict(), stats

    def _stream_packed(self, plan, comps: Dict[str, torch.Tensor]) -> None:
        """Host blocks -> packed staging (one per layout) -> one H2D each ->
        scatter into the component arrays at each block's rows."""
        by_layout: Dict[int, list] = {}
        for dst, rows, host, layout in plan:
            by_layout.setdefault(layout_code(layout), []).append((dst, rows, host))
        for code, items in by_layout.items():
            total = sum(r for _, r, _ in items)
            staging = _pinned_empty((total, 59))
            off = 0
            for _, rows, host in items:
                staging[off:off + rows].copy_(host[:rows])
                off += rows
            packed_gpu = staging.to(self.device, non_blocking=staging.is_pinned())
            tmp = self._alloc_components(total)
            _ops.unpack_rows(packed_gpu, code, tmp, 0)
            src_starts = np.cumsum([0] + [r for _, r, _ in items[:-1]]).tolist()
            _ops.copy_blocks(tmp, None, comps, None, src_starts, [d for d, _, _ in items],
                             [r for _, r, _ in items], self.device)

    def get_retention_stats(self) -> Dict[str, float]:
        total_loaded = self.hotspot_stats["total_blocks_loaded"]
        total_retained = self.hotspot_stats["total_blocks_retained"]
        avg = total_retained / total_loaded if total_loaded > 0 else 0.0
        return {
            "total_iterations": self.hotspot_stats["total_iterations"],
            "avg_hit_rate": avg,
            "total_blocks_loaded": total_loaded,
            "total_blocks_retained": total_retained,
            "total_blocks_cold": self.hotspot_stats["total_blocks_cold"],
            "bandwidth_savings_ratio": avg,
        }

    def update_ram_cache(self, geometry_cache: Dict[str, torch.Tensor], sh_cache: torch.Tensor):
        """Working set -> RAM caches by global id (gpu_working_set.py:795-831)."""
        if self.gpu_xyz is None:
            print("[GPUWorkingSet] Warning: No parameters to update (empty working set)")
            return
        rows = int(self.gpu_xyz.shape[0])
        packed = torch.empty((rows, 59), dtype=torch.float32, device=self.device)
        refs = _ops.pack_rows(self._components(), [0], [rows], packed, _lib.LAYOUT_CACHE)
        host = packed.cpu()
        del refs
        global_ids = self.local_to_global_idx.cpu()
        cols = component_columns("cache")
        for name in ("xyz", "scaling", "rotation", "opacity"):
            geometry_cache[name][global_ids] = host[:, cols[name]]
        sh_cache[global_ids] = host[:, 11:59]

    def get_working_set_size(self) -> Dict[str, float]:
        stats = {"num_gaussians": 0, "memory_mb": 0.0, "num_blocks": len(self.loaded_blocks)}
        if self.gpu_xyz is not None:
            n = int(self.gpu_xyz.shape[0])
            stats["num_gaussians"] = n
            stats["memory_mb"] = n * 59 * 4 / (1024 ** 2)
        return stats

    # ------------------------------------------------------------------
    # Write-back (gpu_working_set.py:852-988)
    # ------------------------------------------------------------------
    def _acquire_writeback_staging(self, required_rows: int):
        slot_idx = self._next_writeback_slot
        self._next_writeback_slot = (slot_idx + 1) % len(self._writeback_staging_slots)
        available = self._writeback_slot_available[slot_idx]
        available.wait()
        available.clear()
        staging = self._writeback_staging_slots[slot_idx]
        gpu_staging = self._writeback_gpu_staging_slots[slot_idx]
        if (staging is not None and gpu_staging is not None
                and required_rows <= self._writeback_staging_capacities[slot_idx]):
            return staging, gpu_staging, available
        # Page-locking a GB-sized buffer takes hundreds of ms: grow
        # geometrically so a write-back set that grows over the first
        # iterations re-allocates O(log) times instead of on every new maximum.
        previous = self._writeback_staging_capacities[slot_idx]
        capacity = max(required_rows, 2 * previous)
        self._writeback_staging_slots[slot_idx] = None
        self._writeback_gpu_staging_slots[slot_idx] = None
        staging = _pinned_empty((capacity, 59))
        gpu_staging = torch.empty((capacity, 59), dtype=torch.float32, device=self.device)
        self._writeback_staging_slots[slot_idx] = staging
        self._writeback_gpu_staging_slots[slot_idx] = gpu_staging
        self._writeback_staging_capacities[slot_idx] = capacity
        self.writeback_stats["pinned_staging_bytes"] = sum(
            s.numel() * s.element_size() for s in self._writeback_staging_slots if s is not None)
        self.writeback_stats["pinned_staging"] = all(
            s.is_pinned() for s in self._writeback_staging_slots if s is not None)
        return staging, gpu_staging, available

    def stage_updated_blocks(self, updated_block_ids: List[int],
                             host_cache=None) -> Optional[PendingBlockWriteback]:
        """Pack updated blocks and enqueue one batched D2H copy. With a
        `host_cache` (PinnedBlockCache) each block's rows go by DMA straight
        into a fresh cache entry instead (PendingCacheWriteback)."""
        sources = self._components()
        if not updated_block_ids or any(t is None for t in sources.values()):
            return None
        plans = []
        src_starts = []
        for block_id in sorted(set(int(b) for b in updated_block_ids)):
            local_slice = self.block_to_gpu_slice.get(block_id)
            if local_slice is None:
                continue
            expected_rows = min(self.block_size, self.num_total - block_id * self.block_size)
            row_count = min(expected_rows, int(local_slice.stop - local_slice.start))
            if row_count <= 0:
                continue
            plans.append((block_id, row_count))
            src_starts.append(int(local_slice.start))
        if not plans:
            return None
        if host_cache is not None:
            return self._stage_into_cache(plans, src_starts, sources, host_cache)
        total_rows = sum(r for _, r in plans)
        staging, gpu_staging, release_event = self._acquire_writeback_staging(total_rows)
        pinned = bool(self.writeback_stats["pinned_staging"])
        packed_cpu = staging[:total_rows]
        packed_gpu = gpu_staging[:total_rows]
        ready_event = torch.cuda.Event()
        current = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self._writeback_stream):
            self._writeback_stream.wait_stream(current)
            refs = _ops.pack_rows(sources, src_starts, [r for _, r in plans], packed_gpu,
                                  _lib.LAYOUT_CACHE)
            packed_cpu.copy_(packed_gpu, non_blocking=pinned)
            ready_event.record(self._writeback_stream)
        for t in sources.values():
            t.record_stream(self._writeback_stream)
        self.writeback_stats["batched_writebacks"] += 1
        self.writeback_stats["batched_writeback_blocks"] += len(plans)
        self.writeback_stats["batched_writeback_rows"] += total_rows
        self.writeback_stats["async_d2h_calls"] += 1
        return PendingBlockWriteback(plans, packed_cpu, ready_event, release_event=release_event,
                                     gpu_refs=[packed_gpu, *refs])

    def ensure_direct_writeback_capacity(self, rows: int) -> torch.Tensor:
        """Device staging of the direct (host-cache) write-back, grown
        geometrically and allocated on the write-back stream, so that a
        regrown buffer is not handed out again before the DMAs reading the
        old one ran; call it once with the largest batch to keep device
        allocations out of the steps."""
        cur = self._direct_staging
        if cur is None or cur.shape[0] < rows:
            capacity = max(int(rows), 2 * (0 if cur is None else int(cur.shape[0])))
            with torch.cuda.stream(self._writeback_stream):
                self._direct_staging = torch.empty((capacity, 59), dtype=torch.float32,
                                                   device=self.device)
        return self._direct_staging

    def _stage_into_cache(self, plans, src_starts, sources, host_cache) -> PendingCacheWriteback:
        total_rows = sum(r for _, r in plans)
        views = host_cache.reserve_writeback(plans)
        ready_event = torch.cuda.Event()
        current = torch.cuda.current_stream(self.device)
        row_bytes = 59 * 4
        try:
            with torch.cuda.stream(self._writeback_stream):
                self._writeback_stream.wait_stream(current)
                packed_gpu = self.ensure_direct_writeback_capacity(total_rows)[:total_rows]
                counts = [r for _, r in plans]
                refs = _ops.pack_rows(sources, src_starts, counts, packed_gpu, _lib.LAYOUT_CACHE)
                offsets = np.concatenate([[0], np.cumsum(counts[:-1])]).astype(np.int64)
                src = (packed_gpu.data_ptr() + offsets * row_bytes).tolist()
                _ops.d2h_blocks([v.data_ptr() for v in views], src,
                                [r * row_bytes for r in counts], self.device)
                ready_event.record(self._writeback_stream)
        except BaseException:
            host_cache.abort_writeback(views)
            raise
        for t in sources.values():
            t.record_stream(self._writeback_stream)
        self.writeback_stats["batched_writebacks"] += 1
        self.writeback_stats["batched_writeback_blocks"] += len(plans)
        self.writeback_stats["batched_writeback_rows"] += total_rows
        self.writeback_stats["direct_cache_d2h_blocks"] += len(plans)
        return PendingCacheWriteback(plans, ready_event, host_cache, views,
                                     gpu_refs=[packed_gpu, *refs])

    def stage_block_bounds(self, block_ids: List[int]) -> Optional[PendingBlockBounds]:
        if self.gpu_xyz is None or not block_ids:
            return None
        plans = []
        for block_id in sorted(set(int(b) for b in block_ids)):
            local_slice = self.block_to_gpu_slice.get(block_id)
            if local_slice is None:
                continue
            expected_rows = min(self.block_size, self.num_total - block_id * self.block_size)
            row_count = min(expected_rows, int(local_slice.stop - local_slice.start))
            if row_count > 0:
                plans.append((block_id, int(local_slice.start), row_count))
        if not plans:
            return None
        bounds_gpu = torch.empty((len(plans), 6), dtype=torch.float32, device=self.device)
        bounds_cpu = _pinned_empty((len(plans), 6))
        ready_event = torch.cuda.Event()
        current = torch.cuda.current_stream(self.device)
        with torch.cuda.stream(self._writeback_stream):
            self._writeback_stream.wait_stream(current)
            refs = _ops.block_bounds(self.gpu_xyz, [p[1] for p in plans], [p[2] for p in plans],
                                     bounds_gpu)
            bounds_cpu.copy_(bounds_gpu, non_blocking=bounds_cpu.is_pinned())
            ready_event.record(self._writeback_stream)
        self.gpu_xyz.record_stream(self._writeback_stream)
        del refs
        self.writeback_stats["bounds_updates"] += len(plans)
        return PendingBlockBounds([p[0] for p in plans], bounds_cpu, ready_event,
                                  gpu_bounds=bounds_gpu)

    def clear(self, release_cuda_cache: bool = True):
        self.gpu_xyz = None
        self.gpu_scaling = None
        self.gpu_rotation = None
        self.gpu_opacity = None
        self.gpu_features_dc = None
        self.gpu_features_rest = None
        self.block_to_gpu_slice.clear()
        self.loaded_blocks.clear()
        self.local_to_global_idx = None
        self._block_starts = None
        if release_cuda_cache and torch.cuda.is_available():
            torch.cuda.empty_cache()

    def prepare_for_retention(self):
        if self.gpu_xyz is not None:
            self.gpu_xyz = self.gpu_xyz.detach()
            self.gpu_scaling = self.gpu_scaling.detach()
            self.gpu_rotation = self.gpu_rotation.detach()
            self.gpu_opacity = self.gpu_opacity.detach()
            self.gpu_features_dc = self.gpu_features_dc.detach()
            self.gpu_features_rest = self.gpu_features_rest.detach()
