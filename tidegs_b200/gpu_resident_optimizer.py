"""GPU-resident Adam over resident block slots (drop-in for TideGS's
strategies/tide_engine/gpu_resident_optimizer.py:73-513 `GPUResidentAdam`).

Same constructor, methods, return values, statistics keys and error messages
as the reference. What changes is where the work happens:

* The six per-component Triton launches (:16-70, :474-499) become one fused
  sm_100a launch updating all 59 columns of every touched row
  (`tgs_resident_adam_apply`).
* Row -> (slot, state row) resolution and the per-slot step / bias tables
  (:266-337) run on the device (`tgs_resident_adam_count`); the host reads
  back one int per resident block to build the returned statistics.
* Optimizer moments live in one [slots*block_size, 128] fp32 array: each state
  row holds the 59 (m, v) pairs plus an admission stamp. Re-admitting a block
  bumps its slot's stamp instead of zero-filling the slot (:207-217, :261);
  rows whose stamp is stale read as m = v = 0, which is the reference's cold
  restart without the memset.
"""
from __future__ import annotations

import math
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib, _ops

# Float index of the admission stamp inside a 128-float state row (the first
# word of the float4 owned by lane 31 in the update kernel).
_STAMP_FLOAT = 124


class GPUResidentAdam:
    """Adam with moments stored only for the current resident block set.

    Blocks keep stable state slots while resident. Eviction releases the slot
    and discards its moments; a later admission starts from zero.
    """

    COMPONENT_SPECS = (
        ("xyz", "_xyz", 3, 0),
        ("opacity", "_opacity", 1, 1),
        ("scaling", "_scaling", 3, 2),
        ("rotation", "_rotation", 4, 3),
        ("features_dc", "_features_dc", 3, 4),
        ("features_rest", "_features_rest", 45, 5),
    )
    TOTAL_WIDTH = sum(spec[2] for spec in COMPONENT_SPECS)
    # First column of each group in a 59-wide columns_lr (UNIFIED order),
    # gpu_resident_optimizer.py:160.
    _GROUP_FIRST_COLUMN = (0, 3, 4, 7, 11, 14)

    def __init__(
        self,
        batch_size: int = 1,
        block_size: int = 4096,
        capacity_blocks: int = 0,
        device: str = "cuda",
    ):
        self.batch_size = int(batch_size)
        self.block_size = int(block_size)
        self.capacity_blocks = max(0, int(capacity_blocks))
        self.device = _lib.require_cuda(device, "GPUResidentAdam")
        self.state_mode = "resident_blocks"
        if self.block_size <= 0:
            raise ValueError(f"[GPUResidentAdam] block_size must be positive, got {block_size}")

        # Slot table (host, numpy): the block each optimizer slot holds (-1:
        # free) and the number of consecutive resident sets that block has
        # been in. Admissions take the lowest free slots; slot numbers are
        # private to this class (the update is independent of them).
        self._allocated_slots = 0
        self._slot_block = np.zeros(0, dtype=np.int64)
        self._slot_streak = np.zeros(0, dtype=np.int64)
        self._ended_streaks = [0, 0]  # (sum, count) of residencies that ended
        self._slot_steps = np.zeros(0, dtype=np.int64)         # host mirror of device steps
        self._slot_initialized = np.zeros(0, dtype=bool)
        self._slot_row_counts = np.zeros(0, dtype=np.int64)
        self._slot_stamp = np.zeros(0, dtype=np.uint32)

        # Device state.
        self._state: Optional[torch.Tensor] = None             # [slots*B, 128] fp32
        self._slot_step_dev: Optional[torch.Tensor] = None     # [slots] int32
        self._slot_stamp_dev: Optional[torch.Tensor] = None    # [slots] int32 (uint32 bits)
        self._slot_bias_dev: Optional[torch.Tensor] = None     # [slots, 2] fp32
        self._err = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._step_tables: Dict[Tuple[float, float], Tuple[torch.Tensor, int, bool]] = {}
        self._slot_tables_dirty = False

        # Reusable buffers for the per-position count read-back.
        self._pin_counts: Optional[torch.Tensor] = None
        self._dev_counts: Optional[torch.Tensor] = None
        # per 32-row chunk of the step's rows: (first local row, first state
        # row) when the update can stream the chunk by bulk copies
        self._chunk_table: Optional[torch.Tensor] = None

        self._logical_state_blocks = 0
        self._logical_state_bytes = 0
        self._stats = {
            "state_mode": "resident_blocks",
            "resident_target_blocks": 0,
            "resident_state_blocks": 0,
            "resident_state_bytes": 0,
            "allocated_state_bytes": 0,
            "cold_restarts": 0,
            "state_evictions": 0,
            "optimizer_rows_touched_total": 0,
            "cold_restarted_rows_touched_total": 0,
            "mean_resident_streak": 0.0,
        }

    # ------------------------------------------------------------------
    # Statistics (gpu_resident_optimizer.py:137-147)
    # ------------------------------------------------------------------
    def _physical_state_bytes(self) -> int:
        return int(self._allocated_slots * self.block_size * _lib.STATE_ROW_FLOATS * 4)

    def _update_state_stats(self) -> None:
        held = self._slot_block >= 0
        n_held = int(np.count_nonzero(held))
        self._stats["resident_target_blocks"] = n_held
        self._stats["resident_state_blocks"] = int(self._logical_state_blocks)
        self._stats["resident_state_bytes"] = int(self._logical_state_bytes)
        self._stats["allocated_state_bytes"] = self._physical_state_bytes()
        # mean residency length over ended residencies and the current ones
        total = self._ended_streaks[0] + int(self._slot_streak[held].sum())
        count = self._ended_streaks[1] + n_held
        self._stats["mean_resident_streak"] = float(total) / max(1, count)

    @property
    def _block_to_slot(self) -> Dict[int, int]:
        """{block id: slot} of the resident blocks."""
        slots = np.nonzero(self._slot_block >= 0)[0]
        return dict(zip(self._slot_block[slots].tolist(), slots.tolist()))

    def _slots_of(self, block_ids: np.ndarray) -> np.ndarray:
        """Slot of each block id, -1 where the block is not resident."""
        slots = np.nonzero(self._slot_block >= 0)[0]
        held = self._slot_block[slots]
        order = np.argsort(held)
        held, slots = held[order], slots[order]
        at = np.minimum(np.searchsorted(held, block_ids), max(held.size - 1, 0))
        found = held.size > 0
        hit = (held[at] == block_ids) if found else np.zeros(block_ids.shape, bool)
        return np.where(hit, slots[at] if found else -1, -1)

    # ------------------------------------------------------------------
    # Learning rates (gpu_resident_optimizer.py:149-169)
    # ------------------------------------------------------------------
    def _normalize_columns_lr(self, columns_lr) -> Dict[str, float]:
        if columns_lr is None:
            raise RuntimeError("[GPUResidentAdam] optimizer.columns_lr is required")
        if torch.is_tensor(columns_lr):
            cols = columns_lr.detach().to(device="cpu", dtype=torch.float32)
        else:
            cols = torch.tensor(columns_lr, dtype=torch.float32)
        cols = cols.flatten().contiguous()
        if cols.numel() == 6:
            grouped = cols
        elif cols.numel() == self.TOTAL_WIDTH:
            grouped = cols[list(self._GROUP_FIRST_COLUMN)]
        else:
            raise RuntimeError(
                f"[GPUResidentAdam] Unexpected columns_lr width={cols.numel()}; "
                "expected 6 grouped or 59 expanded entries"
            )
        return {
            name: float(grouped[group_idx].item())
            for name, _, _, group_idx in self.COMPONENT_SPECS
        }

    # ------------------------------------------------------------------
    # Slot storage (gpu_resident_optimizer.py:171-217)
    # ------------------------------------------------------------------
    def _ensure_storage(self, required_slots: int) -> None:
        if required_slots <= self._allocated_slots:
            return
        target = max(required_slots, self.capacity_blocks, max(1, self._allocated_slots * 2))
        old = self._allocated_slots
        B = self.block_size
        # Zero-filled: a zero stamp never matches a live slot stamp (>= 1).
        state = torch.zeros((target * B, _lib.STATE_ROW_FLOATS), dtype=torch.float32,
                            device=self.device)
        step = torch.zeros(target, dtype=torch.int32, device=self.device)
        stamp = torch.zeros(target, dtype=torch.int32, device=self.device)
        bias = torch.ones((target, 2), dtype=torch.float32, device=self.device)
        if old:
            state[: old * B].copy_(self._state)
            step[:old].copy_(self._slot_step_dev)
            stamp[:old].copy_(self._slot_stamp_dev)
            bias[:old].copy_(self._slot_bias_dev)
        self._state, self._slot_step_dev = state, step
        self._slot_stamp_dev, self._slot_bias_dev = stamp, bias
        grow = target - old
        self._slot_block = np.concatenate([self._slot_block, np.full(grow, -1, np.int64)])
        self._slot_streak = np.concatenate([self._slot_streak, np.zeros(grow, np.int64)])
        self._slot_steps = np.concatenate([self._slot_steps, np.zeros(grow, np.int64)])
        self._slot_initialized = np.concatenate([self._slot_initialized, np.zeros(grow, bool)])
        self._slot_row_counts = np.concatenate([self._slot_row_counts, np.zeros(grow, np.int64)])
        self._slot_stamp = np.concatenate([self._slot_stamp, np.zeros(grow, np.uint32)])
        self._allocated_slots = target

    def _upload_slot_tables(self) -> None:
        """Publishes host step / stamp mirrors after (re)admissions."""
        if not self._slot_tables_dirty:
            return
        _ops.upload_into(self._slot_step_dev, self._slot_steps.astype(np.int32))
        _ops.upload_into(self._slot_stamp_dev, self._slot_stamp.view(np.int32))
        self._slot_tables_dirty = False

    def set_resident_blocks(self, block_ids: List[int]) -> None:
        """Makes `block_ids` the resident set (gpu_resident_optimizer.py:
        219-264 semantics): blocks that leave free their slot and drop their
        moments (a state eviction when the slot had been initialized), blocks
        that stay keep slot and moments, blocks that enter take the lowest
        free slots with a new admission stamp, so their rows read as zero
        moments until first touched (a cold restart). Storage grows to
        max(needed, capacity_blocks, 2 * allocated) slots when it runs out."""
        nxt = np.unique(np.asarray(list(block_ids), dtype=np.int64))
        held_slots = np.nonzero(self._slot_block >= 0)[0]
        stays = np.isin(self._slot_block[held_slots], nxt, assume_unique=True)

        # leaving blocks
        gone = held_slots[~stays]
        if gone.size:
            streaks = self._slot_streak[gone]
            self._ended_streaks[0] += int(streaks.sum())
            self._ended_streaks[1] += int(np.count_nonzero(streaks > 0))
            live = gone[self._slot_initialized[gone]]
            self._stats["state_evictions"] += int(live.size)
            self._logical_state_blocks -= int(live.size)
            self._logical_state_bytes -= int(self._slot_row_counts[live].sum()) * (
                self.TOTAL_WIDTH * 2 * 4)
            self._slot_block[gone] = -1
            self._slot_streak[gone] = 0
            self._slot_steps[gone] = 0
            self._slot_initialized[gone] = False
            self._slot_row_counts[gone] = 0
            self._slot_tables_dirty = True
        self._slot_streak[held_slots[stays]] += 1

        # entering blocks, ascending, into the lowest free slots
        entering = np.setdiff1d(nxt, self._slot_block[held_slots[stays]], assume_unique=True)
        self._ensure_storage(int(nxt.size))
        free = np.nonzero(self._slot_block < 0)[0]
        if free.size < entering.size:
            self._ensure_storage(self._allocated_slots + int(entering.size - free.size))
            free = np.nonzero(self._slot_block < 0)[0]
        if entering.size:
            new = free[: entering.size]
            self._slot_block[new] = entering
            self._slot_streak[new] = 1
            self._slot_steps[new] = 0
            self._slot_initialized[new] = False
            self._slot_row_counts[new] = 0
            # a new admission epoch: every state row of the slot reads as zero
            stamp = self._slot_stamp[new] + np.uint32(1)
            self._slot_stamp[new] = np.where(stamp == 0, np.uint32(1), stamp)
            self._slot_tables_dirty = True
        self._update_state_stats()

    # ------------------------------------------------------------------
    # Step
    # ------------------------------------------------------------------
    def _step_table(self, beta1: float, beta2: float, needed: int) -> Tuple[torch.Tensor, int]:
        """Device table of (1-b1^t, sqrt(1-b2^t)) in fp32 for t < len, computed
        in double precision as gpu_resident_optimizer.py:327-328 does. Once both
        entries round to 1.0f they stay there, and the table stops growing."""
        key = (float(beta1), float(beta2))
        entry = self._step_tables.get(key)
        if entry is not None and (entry[2] or entry[1] >= needed):
            return entry[0], entry[1]
        length = max(needed, 2 * (entry[1] if entry else 64))
        values = [(0.0, 0.0)]
        saturated = False
        for t in range(1, length):
            b1 = np.float32(1.0 - beta1 ** t)
            ds = np.float32(math.sqrt(1.0 - beta2 ** t))
            values.append((float(b1), float(ds)))
            if b1 == np.float32(1.0) and ds == np.float32(1.0) and t >= 1:
                saturated = True
                break
        table = torch.tensor(values, dtype=torch.float32).to(self.device)
        self._step_tables[key] = (table, len(values), saturated)
        return table, len(values)

    def _working_set_layout(self, manager) -> Tuple[np.ndarray, ...]:
        """(starts, ends, block_ids, slots) of loaded blocks sorted by slice
        start (gpu_resident_optimizer.py:266-287)."""
        block_to_slice = manager.block_to_gpu_slice
        rows = []
        for block_id in manager.loaded_blocks:
            block_slice = block_to_slice.get(int(block_id))
            if block_slice is not None:
                rows.append((int(block_slice.start), int(block_slice.stop), int(block_id)))
        if not rows:
            raise RuntimeError("[GPUResidentAdam] working set contains no resident blocks")
        arr = np.asarray(rows, dtype=np.int64)
        slots = self._slots_of(arr[:, 2])
        if np.any(slots < 0):
            missing = int(arr[np.nonzero(slots < 0)[0][0], 2])
            raise RuntimeError(
                f"[GPUResidentAdam] loaded block {missing} has no resident state slot"
            )
        order = np.argsort(arr[:, 0], kind="stable")
        arr, slots = arr[order], slots[order]
        starts, ends = arr[:, 0], arr[:, 1]
        if np.any(ends < starts) or np.any(starts[1:] < ends[:-1]):
            raise RuntimeError("[GPUResidentAdam] resident block slices overlap")
        return starts, ends, arr[:, 2], slots

    def _stage_layout(self, starts, ends, slots) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Device copies of the layout tables, uploaded by kernels on the
        current stream (never queued behind bulk DMA on the copy engines)."""
        P = int(starts.shape[0])
        if self._pin_counts is None or self._pin_counts.numel() < P + 4:
            cap = max(P, 64)
            self._pin_counts = torch.empty(cap + 4, dtype=torch.int32, pin_memory=True)
            self._dev_counts = torch.empty(cap, dtype=torch.int32, device=self.device)
        bounds = _ops.i64_to_device(np.concatenate([starts, ends]), self.device)
        dev_slots = torch.empty(P, dtype=torch.int32, device=self.device)
        _ops.upload_into(dev_slots, np.asarray(slots, dtype=np.int32))
        return bounds[:P], bounds[P:], dev_slots

    def step(
        self,
        iteration: int,
        gaussians,
        sparse_grad_local_ids: torch.Tensor,
        sparse_grad_components: Dict[str, torch.Tensor],
    ) -> Dict[str, Any]:
        if sparse_grad_components is None:
            return self._empty()
        return self._step(iteration, gaussians, sparse_grad_local_ids, sparse_grad_components,
                          None)

    def step_pulled(self, iteration: int, gaussians, sparse_grad_local_ids: torch.Tensor,
                    pull, plan) -> Dict[str, Any]:
        """Multi-GPU step of a block owner (no counterpart in the single-GPU
        reference): the gradient of each row is summed, in rank order, from
        the gradient buffers of the ranks that rendered its block, inside the
        update kernel (sharded.PeerGradPull; plan = the step's ExchangePlan,
        sparse_grad_local_ids = the rows of plan.out_blocks, block_size rows
        each, ascending). Same result and return value as step() given the
        rank-order sum of the contributions."""
        if sparse_grad_local_ids is not None and sparse_grad_local_ids.numel() != (
                plan.n_out * self.block_size):
            raise ValueError(
                f"[GPUResidentAdam] {sparse_grad_local_ids.numel()} rows for "
                f"{plan.n_out} exchanged blocks of {self.block_size}")
        return self._step(iteration, gaussians, sparse_grad_local_ids, None, (pull, plan))

    @staticmethod
    def _empty() -> Dict[str, Any]:
        return {"updated_blocks": 0, "updated_block_ids": [], "touched_rows": 0, "cold_rows": 0}

    def _step(self, iteration, gaussians, sparse_grad_local_ids, sparse_grad_components,
              pulled) -> Dict[str, Any]:
        empty = self._empty()
        if sparse_grad_local_ids is None:
            return empty
        if sparse_grad_local_ids.numel() == 0:
            return empty

        manager = getattr(gaussians, "gpu_working_set_manager", None)
        if manager is None or manager.local_to_global_idx is None:
            raise RuntimeError(
                "[GPUResidentAdam] gpu_working_set_manager with local_to_global_idx is required"
            )
        local_rows = sparse_grad_local_ids.to(device=self.device, dtype=torch.long).contiguous()
        starts, ends, layout_blocks, layout_slots = self._working_set_layout(manager)

        component_lrs = self._normalize_columns_lr(
            getattr(gaussians.optimizer, "columns_lr", None)
        )
        beta1, beta2 = gaussians.optimizer.param_groups[0]["betas"]
        beta1 = float(beta1)
        beta2 = float(beta2)
        eps = float(gaussians.optimizer.param_groups[0]["eps"])

        n = int(local_rows.numel())
        params: List[torch.Tensor] = []
        grads: List[torch.Tensor] = []
        param_rows = None
        for name, attr_name, width, _ in self.COMPONENT_SPECS:
            if pulled is None and name not in sparse_grad_components:
                raise KeyError(
                    f"[GPUResidentAdam] Missing sparse_grad_components[{name!r}] "
                    f"at iter={iteration}"
                )
            param = getattr(gaussians, attr_name).data
            # a pulled step reads the senders' gradients inside the kernel
            grad = None if pulled is not None else sparse_grad_components[name]
            tensors = (param,) if grad is None else (param, grad)
            if not all(t.is_contiguous() for t in tensors):
                raise RuntimeError(
                    f"[GPUResidentAdam] {name} parameter and gradient must be contiguous"
                )
            if any(t.dtype != torch.float32 for t in tensors):
                raise RuntimeError(f"[GPUResidentAdam] {name} must be float32")
            if any(t.device != self.device for t in tensors):
                raise RuntimeError(f"[GPUResidentAdam] {name} must live on {self.device}")
            rows = param.numel() // width
            if param.numel() != rows * width or (grad is not None and grad.numel() != n * width):
                raise RuntimeError(
                    f"[GPUResidentAdam] {name} has shape {tuple(param.shape)} / gradient "
                    f"{None if grad is None else tuple(grad.shape)}; "
                    f"expected [M, {width}] / [{n}, {width}]"
                )
            if param_rows is None:
                param_rows = rows
            elif rows != param_rows:
                raise RuntimeError("[GPUResidentAdam] parameter components differ in row count")
            params.append(param)
            grads.append(grad)

        P = int(starts.shape[0])
        max_step = int(self._slot_steps.max()) if self._slot_steps.size else 0
        table, table_len = self._step_table(beta1, beta2, max_step + 2)
        self._upload_slot_tables()
        pos_start, pos_end, pos_slot = self._stage_layout(starts, ends, layout_slots)
        stream = _lib.stream_handle(self.device)

        chunks = (n + 31) // 32
        if self._chunk_table is None or self._chunk_table.numel() < 2 * chunks:
            self._chunk_table = torch.empty(2 * max(chunks, 1024), dtype=torch.int64,
                                            device=self.device)
        cargs = _lib.ResidentCountArgs(
            pos_start=pos_start.data_ptr(), pos_end=pos_end.data_ptr(),
            pos_slot=pos_slot.data_ptr(), n_positions=P, block_size=self.block_size,
            param_rows=int(param_rows), local_ids=local_rows.data_ptr(), n_rows=n,
            slot_step=self._slot_step_dev.data_ptr(), slot_stamp=self._slot_stamp_dev.data_ptr(),
            slot_bias=self._slot_bias_dev.data_ptr(), step_table=table.data_ptr(),
            step_table_len=table_len, n_slots=self._allocated_slots,
            pos_count=self._dev_counts.data_ptr(), err=self._err.data_ptr(),
            chunk_table=self._chunk_table.data_ptr(),
        )
        _lib.call("tgs_resident_adam_count", cargs, stream)
        # Read back per-position counts + the error word while the update runs.
        pin = self._pin_counts
        pin[:P].copy_(self._dev_counts[:P], non_blocking=True)
        pin[P:P + 4].copy_(self._err, non_blocking=True)
        counts_ready = torch.cuda.Event()
        counts_ready.record(torch.cuda.current_stream(self.device))

        aargs = _lib.ResidentAdamArgs()
        for c, (p, g) in enumerate(zip(params, grads)):
            aargs.param[c] = p.data_ptr()
            aargs.grad[c] = None if g is None else g.data_ptr()
        for c, (name, _, _, _) in enumerate(self.COMPONENT_SPECS):
            aargs.lr[c] = component_lrs[name]
        aargs.beta1, aargs.beta2, aargs.eps = beta1, beta2, eps
        aargs.one_minus_beta1, aargs.one_minus_beta2 = 1.0 - beta1, 1.0 - beta2
        aargs.batch_size = float(self.batch_size)
        aargs.pos_start, aargs.pos_end = pos_start.data_ptr(), pos_end.data_ptr()
        aargs.pos_slot, aargs.n_positions = pos_slot.data_ptr(), P
        aargs.block_size = self.block_size
        aargs.local_ids, aargs.n_rows = local_rows.data_ptr(), n
        aargs.state = self._state.data_ptr()
        aargs.slot_stamp = self._slot_stamp_dev.data_ptr()
        aargs.slot_bias = self._slot_bias_dev.data_ptr()
        aargs.err = self._err.data_ptr()
        aargs.chunk_table = self._chunk_table.data_ptr()
        if pulled is None:
            _lib.call("tgs_resident_adam_apply", aargs, stream)
        else:
            pull, plan = pulled
            pull.apply(aargs, plan, stream)
        counts_ready.synchronize()
        host = pin.numpy()
        problem = _lib.decode_device_error(host[P:P + 4])
        if problem is not None:
            raise RuntimeError(f"[GPUResidentAdam] invalid sparse_grad_local_ids: {problem}")
        counts = host[:P].astype(np.int64)

        touched = np.nonzero(counts > 0)[0]
        t_slots = layout_slots[touched]
        t_counts = counts[touched]
        cold = ~self._slot_initialized[t_slots]
        cold_slots = t_slots[cold]
        cold_rows = int(t_counts[cold].sum())
        cold_row_counts = (ends - starts)[touched][cold]
        self._slot_initialized[cold_slots] = True
        self._slot_row_counts[cold_slots] = cold_row_counts
        self._logical_state_blocks += int(cold.sum())
        self._logical_state_bytes += int(cold_row_counts.sum()) * self.TOTAL_WIDTH * 2 * 4
        self._stats["cold_restarts"] += int(cold.sum())
        self._stats["cold_restarted_rows_touched_total"] += cold_rows
        self._slot_steps[t_slots] += 1

        self._stats["optimizer_rows_touched_total"] += n
        self._update_state_stats()
        touched_blocks = [int(b) for b in layout_blocks[touched]]
        return {
            "updated_blocks": len(touched_blocks),
            "updated_block_ids": touched_blocks,
            "touched_rows": n,
            "cold_rows": cold_rows,
        }

    def get_stats(self) -> Dict[str, Any]:
        self._update_state_stats()
        return dict(self._stats)

    # ------------------------------------------------------------------
    # Inspection (not in the reference API): moments of a resident block.
    # ------------------------------------------------------------------
    def export_block_state(self, block_id: int, rows: Optional[int] = None):
        """Returns ({name: exp_avg}, {name: exp_avg_sq}) for the rows of a
        resident block, with rows untouched since admission reported as zero."""
        slot = self._block_to_slot.get(int(block_id))
        if slot is None:
            raise KeyError(f"[GPUResidentAdam] block {block_id} is not resident")
        B = self.block_size
        rows = B if rows is None else int(rows)
        state = self._state[slot * B: slot * B + rows]
        stamp = int(self._slot_stamp[slot])
        fresh = state[:, _STAMP_FLOAT].view(torch.int32) == np.int32(np.uint32(stamp).view(np.int32))
        pairs = state[:, : 2 * self.TOTAL_WIDTH].reshape(rows, self.TOTAL_WIDTH, 2)
        pairs = torch.where(fresh[:, None, None], pairs, torch.zeros_like(pairs))
        exp_avg, exp_avg_sq = {}, {}
        col = 0
        for name, _, width, _ in self.COMPONENT_SPECS:
            exp_avg[name] = pairs[:, col:col + width, 0].clone()
            exp_avg_sq[name] = pairs[:, col:col + width, 1].clone()
            col += width
        return exp_avg, exp_avg_sq
