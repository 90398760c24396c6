"""The reference's CPU path for one resident-block step -- test infrastructure
only. bench.py times it (its reference arm and its cpu_baseline leg); nothing
in the product imports it.

With `triton = None` TideGS runs every part of the step through torch ops on
whatever device its tensors live on. This class performs those same torch
operations on CPU tensors, in the engine's order for one iteration of
BASELINE configs[3] (strategies/tide_engine/engine.py:2698-2990):

  1. optimizer: `_working_set_state_rows` (searchsorted over the slice
     layout, unique_consecutive, one host read, gpu_resident_optimizer.py:
     266-300), the per-slot step / bias tables (:302-337) and, per
     component, `_vectorized_component_step` (:339-364);
  2. `mark_dirty_blocks` (double_buffer_gpu.py:494-508) and the bounds of the
     updated blocks by `amin`/`amax` per block (gpu_working_set.py:1046-1050);
  3. `dirty_blocks_for_eviction` (double_buffer_gpu.py:510-523) and the
     write-back pack, one `torch.cat` of the six components per block into
     the staging rows, then the copy to the host staging
     (gpu_working_set.py:968-975);
  4. materialization of the incoming blocks: `_pack_streamed_blocks`
     (`torch.cat` of the reader's blocks into the host staging,
     double_buffer_gpu.py:791-809), the staging copy (:1053), the unpack by
     six column-slice copies (:1054-1062), `_fill_streamed_global_ids`
     (:944-951), then the persistent-slot swap `_copy_resident_blocks`
     (seven copies per block, :824-837);
  5. the optimizer's admission of the incoming blocks: their slots' moments
     zero-filled (`set_resident_blocks` + `_clear_slots`, :219-264).

The arithmetic of step 1 is the reference fallback's (oracle/resident_adam.py
pins it bit for bit against the reference's own output); the data movement
is plain copies. Shapes, orders and ops follow the cited lines; the
bookkeeping around them (Python dicts and sets of the drop-in classes) is
left out, which only makes this baseline faster than the reference.
"""
from __future__ import annotations

import math
from typing import Dict, Sequence

import numpy as np
import torch

# (name, width) in the working set's SoA order and in CACHE column order
COMPONENTS = (("xyz", 3), ("opacity", 1), ("scaling", 3), ("rotation", 4),
              ("features_dc", 3), ("features_rest", 45))
CACHE_ORDER = ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest")
CACHE_COLS = {"xyz": (0, 3), "scaling": (3, 6), "rotation": (6, 10), "opacity": (10, 11),
              "features_dc": (11, 14), "features_rest": (14, 59)}
LRS = {"xyz": 1.6e-4, "opacity": 0.05, "scaling": 5e-3, "rotation": 1e-3,
       "features_dc": 2.5e-3, "features_rest": 1.25e-4}


def host_bytes(slots: int, block_size: int, turnover: int, visible_frac: float,
               pool_blocks: int) -> int:
    """Host memory the step holds, for sizing it to the machine."""
    row = 59 * 4
    rows = slots * block_size
    return int(rows * (3 * row + 8)                        # params, m, v, ids
               + turnover * block_size * (4 * row + 8)     # loading, staging x2, wb
               + visible_frac * 1.2 * rows * (row + 16)    # grads, row ids
               + pool_blocks * block_size * row)


class ReferenceCpuStep:
    """Holds the working set, the optimizer state and the staging buffers of
    one rank on the CPU and runs configs[3] iterations over them."""

    def __init__(self, slots: int, block_size: int, turnover: int, max_visible_rows: int,
                 pool_blocks: int = 32, num_blocks: int = 0, seed: int = 0,
                 batch_size: int = 16, betas=(0.9, 0.999), eps: float = 1e-15):
        gen = torch.Generator().manual_seed(seed)
        self.slots, self.B, self.turnover = int(slots), int(block_size), int(turnover)
        self.batch_size, self.betas, self.eps = int(batch_size), tuple(betas), float(eps)
        rows = self.slots * self.B
        # seeded N(0,1) host blocks; block b of the scene holds pool[b % len]
        # (the RNG is serial, so the large buffers are filled from the pool
        # with parallel copies instead of drawing every value)
        self.pool = torch.randn((pool_blocks, self.B, 59), generator=gen)

        def filled(n_rows, name, scale=None):
            a, z = CACHE_COLS[name]
            out = torch.empty((n_rows, z - a))
            for i in range(0, n_rows, self.B):
                k = min(self.B, n_rows - i)
                out[i:i + k].copy_(self.pool[(i // self.B) % pool_blocks, :k, a:z])
            return out.mul_(scale) if scale is not None else out

        def zeros(*shape, dtype=torch.float32):
            return torch.empty(shape, dtype=dtype).fill_(0)  # parallel first touch

        self.params = {n: filled(rows, n) for n, _ in COMPONENTS}
        self.local_to_global = zeros(rows, dtype=torch.long)
        self.exp_avg = {n: zeros(rows, w) for n, w in COMPONENTS}
        self.exp_avg_sq = {n: zeros(rows, w) for n, w in COMPONENTS}
        self.slot_steps = [0] * self.slots
        self.bias1 = torch.ones(self.slots)
        self.denom_scale = torch.ones(self.slots)
        self.grads = {n: filled(max_visible_rows, n, 1e-3) for n, _ in COMPONENTS}
        lrows = self.turnover * self.B
        self.loading = {n: zeros(lrows, w) for n, w in COMPONENTS}
        self.loading_gids = zeros(lrows, dtype=torch.long)
        self.staging_cpu = zeros(lrows, 59)
        self.staging_dev = zeros(lrows, 59)
        self.wb_dev = zeros(lrows, 59)
        self.wb_cpu = zeros(lrows, 59)
        self.num_blocks = max(int(num_blocks), 1)
        self.dirty = torch.zeros(self.num_blocks, dtype=torch.bool)
        # slice layout: position p holds rows [p*B, (p+1)*B); a block's state
        # slot is its position (any fixed assignment times the same)
        self.starts = torch.arange(self.slots, dtype=torch.long) * self.B
        self.ends = self.starts + self.B
        self.slot_of_pos = torch.arange(self.slots, dtype=torch.long)

    # -- 1. optimizer ---------------------------------------------------------
    def adam(self, local_ids: torch.Tensor) -> int:
        beta1, beta2 = self.betas
        pos = torch.searchsorted(self.ends, local_ids, right=True)
        state_slots = self.slot_of_pos[pos]
        state_rows = state_slots * self.B + (local_ids - self.starts[pos])
        touched, _counts = torch.unique_consecutive(pos, return_counts=True)
        touched_slots = self.slot_of_pos[touched].tolist()
        bias, denom = [], []
        for s in touched_slots:
            self.slot_steps[s] += 1
            t = self.slot_steps[s]
            bias.append(1.0 - beta1 ** t)
            denom.append(math.sqrt(1.0 - beta2 ** t))
        idx = torch.tensor(touched_slots, dtype=torch.long)
        self.bias1.index_copy_(0, idx, torch.tensor(bias, dtype=torch.float32))
        self.denom_scale.index_copy_(0, idx, torch.tensor(denom, dtype=torch.float32))
        n = int(local_ids.numel())
        for name, _ in COMPONENTS:
            param, m, v = self.params[name], self.exp_avg[name], self.exp_avg_sq[name]
            grad = self.grads[name][:n]
            avg = m.index_select(0, state_rows)
            avg_sq = v.index_select(0, state_rows)
            g = grad / float(self.batch_size)
            avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
            avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
            m.index_copy_(0, state_rows, avg)
            v.index_copy_(0, state_rows, avg_sq)
            b = self.bias1.index_select(0, state_slots).unsqueeze(1)
            ds = self.denom_scale.index_select(0, state_slots).unsqueeze(1)
            update = (avg / (avg_sq.sqrt() / ds + self.eps)) * (LRS[name] / b)
            param.index_copy_(0, local_ids, param.index_select(0, local_ids) - update)
        return n

    # -- one iteration ----------------------------------------------------------
    def step(self, local_ids: torch.Tensor, updated_blocks: Sequence[int],
             updated_pos: Sequence[int], evict_pos: np.ndarray, evicted_blocks: np.ndarray,
             incoming_blocks: np.ndarray, dirty_pattern: np.ndarray) -> int:
        B = self.B
        n = self.adam(local_ids)
        # 2. dirty marks and bounds of the updated blocks
        ids = torch.tensor(sorted(set(int(b) % self.num_blocks for b in updated_blocks)),
                           dtype=torch.long)
        self.dirty.index_fill_(0, ids, True)
        bounds = torch.empty((len(updated_pos), 6))
        xyz = self.params["xyz"]
        for i, p in enumerate(updated_pos):
            rows = xyz[int(p) * B:(int(p) + 1) * B]
            bounds[i, :3] = rows.amin(dim=0)
            bounds[i, 3:] = rows.amax(dim=0)
        # 3. dirty-and-evicted selection and the write-back pack
        ev = np.asarray(evicted_blocks, np.int64) % self.num_blocks
        if dirty_pattern is not None:
            # a prescribed dirty pattern instead of the updates
            self.dirty.index_fill_(0, torch.from_numpy(ev[dirty_pattern]), True)
            self.dirty.index_fill_(0, torch.from_numpy(ev[~dirty_pattern]), False)
        order = np.argsort(ev, kind="stable")
        ev_t = torch.from_numpy(ev[order])
        selected = ev_t[self.dirty.index_select(0, ev_t)].tolist()
        sel = set(selected)
        wb_pos = [int(p) for p, b in zip(np.asarray(evict_pos)[order], ev[order]) if int(b) in sel]
        off = 0
        for p in wb_pos:
            sl = slice(p * B, (p + 1) * B)
            self.wb_dev[off:off + B] = torch.cat([self.params[c][sl] for c in CACHE_ORDER], dim=1)
            off += B
        self.wb_cpu[:off].copy_(self.wb_dev[:off])
        self.dirty.index_fill_(0, torch.tensor(selected, dtype=torch.long), False)
        # 4. materialization of the incoming blocks, then the slot swap
        k = len(incoming_blocks)
        pieces = [self.pool[int(b) % self.pool.shape[0]] for b in incoming_blocks]
        torch.cat(pieces, dim=0, out=self.staging_cpu[:k * B])
        self.staging_dev[:k * B].copy_(self.staging_cpu[:k * B])
        for name, _ in COMPONENTS:
            a, z = CACHE_COLS[name]
            self.loading[name][:k * B].copy_(self.staging_dev[:k * B, a:z])
        r = torch.arange(k * B, dtype=torch.long)
        blk = torch.div(r, B, rounding_mode="floor")
        inc = torch.as_tensor(np.asarray(incoming_blocks, np.int64))
        self.loading_gids[:k * B] = inc[blk] * B + (r - blk * B)
        for i, p in enumerate(sorted(int(x) for x in evict_pos)):
            src, dst = slice(i * B, (i + 1) * B), slice(p * B, (p + 1) * B)
            for name, _ in COMPONENTS:
                self.params[name][dst].copy_(self.loading[name][src])
            self.local_to_global[dst].copy_(self.loading_gids[src])
        # 5. the incoming blocks' optimizer slots start from zero moments
        rows = (torch.as_tensor(np.asarray(evict_pos, np.int64))[:, None] * B
                + torch.arange(B)[None, :]).reshape(-1)
        for name, _ in COMPONENTS:
            self.exp_avg[name].index_fill_(0, rows, 0.0)
            self.exp_avg_sq[name].index_fill_(0, rows, 0.0)
        for p in evict_pos:
            self.slot_steps[int(p)] = 0
        return n
