"""CPU restatement of TideGS's GPU-resident Adam -- test infrastructure only.

Follows strategies/tide_engine/gpu_resident_optimizer.py:
  slot allocator / eviction / admission   :171-264
  row -> (slot, state row), touched sets  :266-300
  per-slot step and bias tables           :302-337
  per-element update                      :16-70 (kernel)  and :339-364 (torch fallback)

Two arithmetic modes for the per-element update:
  "kernel": the op order of the fused kernel (:47-66) in numpy float32, every
            operation rounded once (no FMA). libtidegs_b200's update is checked
            bit-for-bit against this mode.
  "torch":  the reference's torch CPU fallback op sequence (:353-364), the
            arithmetic the reference runs without Triton. Golden vectors from
            the reference pin this mode; it is also the timed CPU baseline.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

COMPONENT_SPECS = (
    ("xyz", "_xyz", 3, 0),
    ("opacity", "_opacity", 1, 1),
    ("scaling", "_scaling", 3, 2),
    ("rotation", "_rotation", 4, 3),
    ("features_dc", "_features_dc", 3, 4),
    ("features_rest", "_features_rest", 45, 5),
)
TOTAL_WIDTH = 59
F32 = np.float32


def kernel_update(param, grad, m, v, lr, bias1, denom_scale, beta1, beta2, eps, batch_size):
    """Per-element Adam in the fused kernel's order, which is the reference
    torch fallback's order (:355-364) with every operation rounded once:
        g = grad / bs
        m = b1*m + (1-b1)*g          (1-b1 taken in double, then rounded)
        v = b2*v + ((1-b2)*g)*g
        p = p - (m / (sqrt(v)/denom_scale + eps)) * ((1/bias1) * lr)
    All arguments float32 arrays or scalars (bias1/denom_scale broadcast per
    row). Returns (p, m, v)."""
    b1, b2, e, bs = F32(beta1), F32(beta2), F32(eps), F32(batch_size)
    omb1, omb2 = F32(1.0 - float(beta1)), F32(1.0 - float(beta2))
    g = grad / bs
    m = b1 * m + omb1 * g
    v = b2 * v + (omb2 * g) * g
    denom = np.sqrt(v) / denom_scale + e
    scale = (F32(1.0) / bias1) * F32(lr)
    p = param - (m / denom) * scale
    return p.astype(F32), m.astype(F32), v.astype(F32)


def bias_pair(beta1: float, beta2: float, step: int) -> Tuple[np.float32, np.float32]:
    """(1 - b1^t, sqrt(1 - b2^t)) in double, rounded to float32 (:327-336)."""
    return F32(1.0 - beta1 ** step), F32(math.sqrt(1.0 - beta2 ** step))


class ResidentAdamOracle:
    """Host model of GPUResidentAdam's slot bookkeeping plus the update."""

    def __init__(self, batch_size: int = 1, block_size: int = 4096, capacity_blocks: int = 0,
                 arithmetic: str = "kernel"):
        if arithmetic not in ("kernel", "torch"):
            raise ValueError(arithmetic)
        self.batch_size = int(batch_size)
        self.block_size = int(block_size)
        self.capacity_blocks = max(0, int(capacity_blocks))
        self.arithmetic = arithmetic
        self._resident = set()
        self._streaks: Dict[int, int] = {}
        self._done_streak_total = 0
        self._done_streak_count = 0
        self._allocated = 0
        self._block_to_slot: Dict[int, int] = {}
        self._free: List[int] = []
        self._steps: List[int] = []
        self._init: List[bool] = []
        self._rows: List[int] = []
        self.exp_avg: Dict[str, np.ndarray] = {}
        self.exp_avg_sq: Dict[str, np.ndarray] = {}
        self._logical_blocks = 0
        self._logical_bytes = 0
        self.stats = {
            "cold_restarts": 0, "state_evictions": 0, "optimizer_rows_touched_total": 0,
            "cold_restarted_rows_touched_total": 0,
        }

    def _ensure(self, required: int) -> None:
        if required <= self._allocated:
            return
        target = max(required, self.capacity_blocks, max(1, self._allocated * 2))
        old = self._allocated
        B = self.block_size
        for name, _, w, _ in COMPONENT_SPECS:
            for store in (self.exp_avg, self.exp_avg_sq):
                new = np.zeros((target * B, w), F32)
                if old:
                    new[: old * B] = store[name]
                store[name] = new
        grow = target - old
        self._steps += [0] * grow
        self._init += [False] * grow
        self._rows += [0] * grow
        self._free.extend(range(target - 1, old - 1, -1))
        self._allocated = target

    def set_resident_blocks(self, block_ids: Sequence[int]) -> None:
        nxt = {int(b) for b in block_ids}
        prev = set(self._resident)
        evicted, kept, incoming = prev - nxt, prev & nxt, nxt - prev
        for b in evicted:
            streak = int(self._streaks.pop(b, 0))
            if streak > 0:
                self._done_streak_total += streak
                self._done_streak_count += 1
            slot = self._block_to_slot.pop(b)
            if self._init[slot]:
                self.stats["state_evictions"] += 1
                self._logical_blocks -= 1
                self._logical_bytes -= self._rows[slot] * TOTAL_WIDTH * 8
            self._steps[slot] = 0
            self._init[slot] = False
            self._rows[slot] = 0
            self._free.append(slot)
        for b in kept:
            self._streaks[b] = self._streaks.get(b, 0) + 1
        for b in incoming:
            self._streaks[b] = 1
        self._ensure(len(nxt))
        B = self.block_size
        for b in sorted(incoming):
            if not self._free:
                self._ensure(self._allocated + 1)
            slot = self._free.pop()
            self._block_to_slot[b] = slot
            self._steps[slot] = 0
            self._init[slot] = False
            self._rows[slot] = 0
            for store in (self.exp_avg, self.exp_avg_sq):
                for name in store:
                    store[name][slot * B:(slot + 1) * B] = 0.0
        self._resident = nxt

    def resident_state_blocks(self) -> int:
        return self._logical_blocks

    def step(self, params: Dict[str, np.ndarray], local_ids: np.ndarray,
             grads: Dict[str, np.ndarray], layout: Sequence[Tuple[int, slice]],
             columns_lr: Sequence[float], betas=(0.9, 0.999), eps: float = 1e-15) -> dict:
        """Mutates params in place. layout = manager.loaded_blocks order with
        their slices; columns_lr = 6 grouped learning rates."""
        ids = np.asarray(local_ids, np.int64)
        if ids.size == 0:
            return {"updated_blocks": 0, "updated_block_ids": [], "touched_rows": 0,
                    "cold_rows": 0}
        items = []
        for b, sl in layout:
            slot = self._block_to_slot.get(int(b))
            if slot is None:
                raise RuntimeError(f"loaded block {b} has no resident state slot")
            items.append((int(sl.start), int(sl.stop), int(b), slot))
        items.sort(key=lambda it: it[0])
        starts = np.array([it[0] for it in items], np.int64)
        ends = np.array([it[1] for it in items], np.int64)
        slots = np.array([it[3] for it in items], np.int64)
        pos = np.searchsorted(ends, ids, side="right")
        row_in_block = ids - starts[pos]
        state_slots = slots[pos]
        state_rows = state_slots * self.block_size + row_in_block
        touched_pos, counts = np.unique(pos, return_counts=True)  # ids sorted -> consecutive
        beta1, beta2 = float(betas[0]), float(betas[1])
        bias = np.ones(self._allocated, F32)
        dscale = np.ones(self._allocated, F32)
        cold_rows = 0
        for p, cnt in zip(touched_pos.tolist(), counts.tolist()):
            start, stop, b, slot = items[p]
            if not self._init[slot]:
                self._init[slot] = True
                self._rows[slot] = stop - start
                self._logical_blocks += 1
                self._logical_bytes += (stop - start) * TOTAL_WIDTH * 8
                self.stats["cold_restarts"] += 1
                self.stats["cold_restarted_rows_touched_total"] += int(cnt)
                cold_rows += int(cnt)
            self._steps[slot] += 1
            bias[slot], dscale[slot] = bias_pair(beta1, beta2, self._steps[slot])
        lrs = list(columns_lr)
        for name, _, w, gi in COMPONENT_SPECS:
            p_rows = params[name][ids]
            m = self.exp_avg[name][state_rows]
            v = self.exp_avg_sq[name][state_rows]
            g = np.asarray(grads[name], F32).reshape(ids.size, w)
            b1c = bias[state_slots][:, None]
            dsc = dscale[state_slots][:, None]
            if self.arithmetic == "kernel":
                p_new, m, v = kernel_update(p_rows, g, m, v, F32(lrs[gi]), b1c, dsc, beta1, beta2,
                                            eps, self.batch_size)
            else:
                p_new, m, v = torch_fallback_update(p_rows, g, m, v, float(lrs[gi]), b1c, dsc,
                                                    beta1, beta2, eps, self.batch_size)
            self.exp_avg[name][state_rows] = m
            self.exp_avg_sq[name][state_rows] = v
            params[name][ids] = p_new
        self.stats["optimizer_rows_touched_total"] += int(ids.size)
        return {
            "updated_blocks": int(touched_pos.size),
            "updated_block_ids": [items[p][2] for p in touched_pos.tolist()],
            "touched_rows": int(ids.size),
            "cold_rows": cold_rows,
        }


def torch_fallback_update(param, grad, m, v, lr, bias1, denom_scale, beta1, beta2, eps, bs):
    """The reference's torch CPU op sequence (gpu_resident_optimizer.py:353-364)."""
    import torch

    avg = torch.from_numpy(np.ascontiguousarray(m))
    avg_sq = torch.from_numpy(np.ascontiguousarray(v))
    g = torch.from_numpy(np.ascontiguousarray(grad)) / float(bs)
    avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
    avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    b = torch.from_numpy(np.ascontiguousarray(bias1))
    ds = torch.from_numpy(np.ascontiguousarray(denom_scale))
    update = (avg / (avg_sq.sqrt() / ds + eps)) * (lr / b)
    values = torch.from_numpy(np.ascontiguousarray(param)) - update
    return values.numpy(), avg.numpy(), avg_sq.numpy()


# ---------------------------------------------------------------------------
# Timed CPU baseline: the reference fallback's per-component torch step over
# resident slots, using all host threads (gpu_resident_optimizer.py:339-364,
# driven as step() :474-499 drives it).
# ---------------------------------------------------------------------------
class TorchFallbackResidentAdam:
    """Dense-slot variant of the reference CPU path for timing: params and
    moments are torch CPU tensors [rows, W] per component, rows = slots*B."""

    def __init__(self, rows: int, seed: int = 0):
        import torch

        gen = torch.Generator().manual_seed(seed)
        self.params = {n: torch.randn((rows, w), generator=gen) for n, _, w, _ in COMPONENT_SPECS}
        self.exp_avg = {n: torch.zeros((rows, w)) for n, _, w, _ in COMPONENT_SPECS}
        self.exp_avg_sq = {n: torch.zeros((rows, w)) for n, _, w, _ in COMPONENT_SPECS}
        self.bias = None
        self.dscale = None

    def step(self, local_rows, state_rows, state_slots, grads, lrs, n_slots, step=1,
             betas=(0.9, 0.999), eps=1e-15, batch_size=1):
        import torch

        beta1, beta2 = betas
        bias = torch.full((n_slots,), 1.0 - beta1 ** step, dtype=torch.float32)
        dscale = torch.full((n_slots,), math.sqrt(1.0 - beta2 ** step), dtype=torch.float32)
        for name, _, w, gi in COMPONENT_SPECS:
            param = self.params[name]
            avg = self.exp_avg[name].index_select(0, state_rows)
            avg_sq = self.exp_avg_sq[name].index_select(0, state_rows)
            scaled = grads[name] / float(batch_size)
            avg.mul_(beta1).add_(scaled, alpha=1.0 - beta1)
            avg_sq.mul_(beta2).addcmul_(scaled, scaled, value=1.0 - beta2)
            self.exp_avg[name].index_copy_(0, state_rows, avg)
            self.exp_avg_sq[name].index_copy_(0, state_rows, avg_sq)
            b = bias.index_select(0, state_slots).unsqueeze(1)
            ds = dscale.index_select(0, state_slots).unsqueeze(1)
            update = (avg / (avg_sq.sqrt() / ds + eps)) * (lrs[gi] / b)
            values = param.index_select(0, local_rows) - update
            param.index_copy_(0, local_rows, values)
