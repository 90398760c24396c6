"""Generates the golden fixtures of tests/golden/ by running the reference
TideGS hot path (its torch CPU fallbacks) on seeded CPU inputs.

    python tests/golden/make_golden.py --reference <path to the TideGS checkout>

Outputs (committed): resident_adam.npz/.json, double_buffer.npz/.json,
writeback.npz/.json, dirty.json. The fixtures pin the CPU oracle
(oracle/) and are what the GPU parity tests compare against; the reference
itself is not needed to run the tests.
"""
from __future__ import annotations

import argparse
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from reference_shim import load_reference  # noqa: E402

COMPONENTS = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")
WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}
ATTRS = {n: "_" + n for n in COMPONENTS}


def baseline_params(rows: int, gen: torch.Generator):
    """Parameter distributions of the benchmark configs (by component name)."""
    q = torch.randn((rows, 4), generator=gen)
    q = q / q.norm(dim=1, keepdim=True)
    rest = torch.randn((rows, 45), generator=gen) * 0.01
    return {
        "xyz": torch.rand((rows, 3), generator=gen) * 200.0 - 100.0,
        "features_dc": torch.randn((rows, 3), generator=gen) * 0.3,
        "features_rest": rest,
        "opacity": torch.randn((rows, 1), generator=gen) - 2.0,
        "scaling": torch.randn((rows, 3), generator=gen) * 0.5 - 4.0,
        "rotation": q,
    }


class _Manager:
    def __init__(self, layout):
        self.set_layout(layout)

    def set_layout(self, layout):
        self.loaded_blocks = [b for b, _ in layout]
        self.block_to_gpu_slice = {b: s for b, s in layout}
        self.local_to_global_idx = torch.arange(max(s.stop for _, s in layout))


class _Gaussians:
    def __init__(self, manager, params, columns_lr, betas, eps):
        self.gpu_working_set_manager = manager
        self.set_params(params)
        self.optimizer = types.SimpleNamespace(
            columns_lr=torch.tensor(columns_lr, dtype=torch.float32),
            param_groups=[{"betas": betas, "eps": eps}])

    def set_params(self, params):
        for n in COMPONENTS:
            setattr(self, ATTRS[n], torch.nn.Parameter(params[n].clone()))

    def values(self):
        return {n: getattr(self, ATTRS[n]).detach().clone() for n in COMPONENTS}


def resident_adam(gro, out_dir: Path) -> None:
    """Two scenarios: the reference unit-test sequence (block 4) and a medium
    sequence with benchmark-like values, eviction, re-admission and a short
    tail block."""
    arrays, meta = {}, {"scenarios": []}

    def run(name, block_size, batch_size, lrs, betas, eps, capacity, phases, param_fn):
        opt = gro.GPUResidentAdam(batch_size=batch_size, block_size=block_size,
                                  capacity_blocks=capacity, device="cpu")
        sc = {"name": name, "block_size": block_size, "batch_size": batch_size,
              "columns_lr": lrs, "betas": list(betas), "eps": eps, "capacity": capacity,
              "phases": []}
        manager = None
        gaussians = None
        for pi, ph in enumerate(phases):
            layout = [(b, slice(s, e)) for b, s, e in ph["layout"]]
            rows = max(e for _, _, e in ph["layout"])
            params = param_fn(rows, ph["param_seed"])
            if manager is None:
                manager = _Manager(layout)
                gaussians = _Gaussians(manager, params, lrs, betas, eps)
            else:
                manager.set_layout(layout)
                gaussians.set_params(params)
            opt.set_resident_blocks(ph["resident"])
            for n in COMPONENTS:
                arrays[f"{name}/p{pi}/init/{n}"] = params[n].numpy()
            steps = []
            for si, (ids, gseed) in enumerate(ph["steps"]):
                ids_t = torch.tensor(ids, dtype=torch.long)
                gen = torch.Generator().manual_seed(gseed)
                grads = {n: torch.randn((len(ids), WIDTHS[n]), generator=gen) * ph["grad_scale"]
                         for n in COMPONENTS}
                stats = opt.step(iteration=si + 1, gaussians=gaussians,
                                 sparse_grad_local_ids=ids_t, sparse_grad_components=grads)
                arrays[f"{name}/p{pi}/s{si}/ids"] = ids_t.numpy()
                for n in COMPONENTS:
                    arrays[f"{name}/p{pi}/s{si}/grad/{n}"] = grads[n].numpy()
                    arrays[f"{name}/p{pi}/s{si}/out/{n}"] = gaussians.values()[n].numpy()
                steps.append(stats)
            sc["phases"].append({"layout": ph["layout"], "resident": ph["resident"],
                                 "step_stats": steps})
        agg = opt.get_stats()
        sc["final_stats"] = {k: agg[k] for k in ("cold_restarts", "state_evictions",
                                                 "resident_state_blocks",
                                                 "optimizer_rows_touched_total",
                                                 "cold_restarted_rows_touched_total")}
        meta["scenarios"].append(sc)

    def randn_params(rows, seed):
        gen = torch.Generator().manual_seed(seed)
        return {n: torch.randn((rows, WIDTHS[n]), generator=gen) for n in COMPONENTS}

    run("unit", 4, 3, [0.01, 0.02, 0.03, 0.04, 0.05, 0.06], (0.9, 0.999), 1e-15, 2, [
        {"layout": [(10, 0, 4), (20, 4, 7)], "resident": [10, 20], "param_seed": 10,
         "grad_scale": 1.0, "steps": [([0, 2, 4, 6], 20), ([1, 4, 5], 21)]},
        {"layout": [(20, 0, 3), (30, 3, 7)], "resident": [20, 30], "param_seed": 11,
         "grad_scale": 1.0, "steps": [([0, 2, 3, 6], 22)]},
        {"layout": [(10, 0, 4)], "resident": [10], "param_seed": 12, "grad_scale": 1.0,
         "steps": [([0, 3], 23)]},
    ], randn_params)

    B = 64
    rng = np.random.default_rng(7)

    def bern(rows, p=0.3):
        return sorted(np.nonzero(rng.random(rows) < p)[0].tolist())

    def layout_of(order, lengths):
        out, off = [], 0
        for b in order:
            out.append((b, off, off + lengths.get(b, B)))
            off += lengths.get(b, B)
        return out

    tail = {11: 40}  # block 11 is the scene's short last block
    l1 = layout_of([3, 5, 7, 8, 10, 11], tail)
    l2 = layout_of([5, 13, 8, 12, 2], tail)      # slice order != id order
    l3 = layout_of([7, 3, 8, 11], tail)
    rows = lambda lay: max(e for _, _, e in lay)  # noqa: E731
    phases = [
        {"layout": l1, "resident": [3, 5, 7, 8, 10, 11], "param_seed": 100, "grad_scale": 1e-3,
         "steps": [(bern(rows(l1)), 200), (bern(rows(l1)), 201), (bern(rows(l1)), 202)]},
        {"layout": l2, "resident": [2, 5, 8, 12, 13], "param_seed": 101, "grad_scale": 1e-3,
         "steps": [(bern(rows(l2)), 203), (bern(rows(l2)), 204)]},
        {"layout": l3, "resident": [3, 7, 8, 11], "param_seed": 102, "grad_scale": 1e-3,
         "steps": [(bern(rows(l3)), 205), (bern(rows(l3)), 206)]},
    ]

    def base_params(rows_, seed):
        return baseline_params(rows_, torch.Generator().manual_seed(seed))

    run("medium", B, 16, [1.6e-4, 0.05, 5e-3, 1e-3, 2.5e-3, 1.25e-4], (0.9, 0.999), 1e-15, 4,
        phases, base_params)

    np.savez_compressed(out_dir / "resident_adam.npz", **arrays)
    (out_dir / "resident_adam.json").write_text(json.dumps(meta, indent=1))


def _components(global_ids):
    """Value = function of the global id (reference test helper shape)."""
    rows = global_ids.to(dtype=torch.float32).unsqueeze(1)
    return {
        "xyz": rows + torch.tensor([0.1, 0.2, 0.3]),
        "scaling": rows + torch.tensor([1.1, 1.2, 1.3]),
        "rotation": rows + torch.tensor([2.1, 2.2, 2.3, 2.4]),
        "opacity": rows + 3.1,
        "features_dc": rows + torch.tensor([4.1, 4.2, 4.3]),
        "features_rest": rows + torch.arange(45) * 0.01 + 5.0,
    }


def _pack(values, layout_name):
    order = (("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest")
             if layout_name == "cache" else COMPONENTS)
    return torch.cat([values[n] for n in order], dim=1)


class _Reader:
    def __init__(self, br, layout, blocks):
        self._br = br
        self.layout = layout
        self.blocks = blocks
        self.calls = []

    def read_blocks(self, ids):
        self.calls.append(list(ids))
        return {b: self.blocks[b] for b in ids}

    def read_batch(self, ids, out=None):
        return self._br._pack_block_batch(self.read_blocks(ids), ids, self.layout, out)


def _buffer_record(prefix, buf, arrays):
    # copies: the reference keeps mutating these tensors in place afterwards
    for n in COMPONENTS:
        arrays[f"{prefix}/{n}"] = getattr(buf, n).numpy().copy()
    arrays[f"{prefix}/gids"] = buf.local_to_global_idx.numpy().copy()
    arrays[f"{prefix}/block_starts"] = buf._block_starts.numpy().copy()
    return {
        "loaded_blocks": [int(b) for b in buf.loaded_blocks],
        "resident_blocks": [int(b) for b in buf.resident_blocks],
        "streamed_blocks": [int(b) for b in buf.streamed_blocks],
        "evicted_blocks": [int(b) for b in buf.evicted_blocks],
        "slices": {str(b): [s.start, s.stop] for b, s in buf.block_to_local_slice.items()},
    }


def double_buffer(br, dbuf, out_dir: Path) -> None:
    arrays, meta = {}, {}
    DB = dbuf.DoubleBufferGPUWorkingSet
    # (1) reference unit-test layouts: resident [1,3] (3 is the short tail), streamed [2].
    for lname, layout in (("cache", br.BlockLayout.CACHE), ("unified", br.BlockLayout.UNIFIED)):
        m = DB(num_total_gaussians=14, block_size=4, device="cpu", verbose=False)
        src_ids = torch.tensor([4, 5, 6, 7, 12, 13])
        vals = _components(src_ids)
        s = m.active_buffer
        for n in COMPONENTS:
            setattr(s, n, vals[n])
        s.local_to_global_idx = src_ids
        s.loaded_blocks = [1, 3]
        s.block_to_local_slice = {1: slice(0, 4), 3: slice(4, 6)}
        s.num_gaussians = 6
        reader = _Reader(br, layout, {2: _pack(_components(torch.tensor([8, 9, 10, 11])), lname)})
        m.start_prefetch(iteration=17, visible_block_ids=[3, 2, 1], resident_block_ids=[1, 3],
                         evicted_block_ids=[0], block_reader=reader)
        assert m.wait_for_prefetch(17)
        rec = _buffer_record(f"unit_{lname}/loading", m.loading_buffer, arrays)
        st = m.get_stats()
        rec["stats"] = {k: st[k] for k in ("batched_materializations", "batched_h2d_calls",
                                           "batched_resident_blocks", "batched_streamed_blocks")}
        rec["reader_calls"] = reader.calls
        for n in COMPONENTS:
            getattr(s, n).add_(10.0)
        h = m.finalize_retained_blocks([1, 3], target="loading")
        rec["handoff"] = [h.ready_blocks, h.copied_blocks]
        for n in COMPONENTS:
            arrays[f"unit_{lname}/refreshed/{n}"] = getattr(m.loading_buffer, n).numpy().copy()
        m.swap_buffers()
        rec["global_to_local_4_12_8"] = m.global_to_local(torch.tensor([4, 12, 8])).tolist()
        meta[f"unit_{lname}"] = rec
        m.clear()

    # (2) random blocks, A/B fallback path with a resident copy and a tail block.
    B, nblocks, tail = 16, 20, 11
    num_total = (nblocks - 1) * B + tail
    gen = torch.Generator().manual_seed(5)
    scene = torch.randn((num_total, 59), generator=gen)   # CACHE layout rows of every block
    blocks = {b: scene[b * B: min((b + 1) * B, num_total)].clone() for b in range(nblocks)}
    m = DB(num_total_gaussians=num_total, block_size=B, device="cpu", verbose=False)
    s = m.active_buffer
    active = [0, 2, 4, 6]
    rows = torch.cat([blocks[b] for b in active])
    cols = {"xyz": (0, 3), "scaling": (3, 6), "rotation": (6, 10), "opacity": (10, 11),
            "features_dc": (11, 14), "features_rest": (14, 59)}
    for n, (a, b_) in cols.items():
        setattr(s, n, (rows[:, a:b_] + 1000.0).contiguous())  # distinguishable from the pool
    s.local_to_global_idx = torch.cat([torch.arange(b * B, b * B + B) for b in active])
    s.loaded_blocks = list(active)
    s.block_to_local_slice = {b: slice(i * B, (i + 1) * B) for i, b in enumerate(active)}
    s.num_gaussians = len(active) * B
    reader = _Reader(br, br.BlockLayout.CACHE, blocks)
    filt = torch.tensor([2 * B + 3, 7 * B, 5 * B + 1, 19 * B + 10, 19 * B + 12, -5, 4 * B + 15])
    m.start_prefetch(iteration=3, visible_block_ids=[7, 4, 2, 19, 3], filters_global=[filt],
                     resident_block_ids=[2, 4], evicted_block_ids=[0, 6], block_reader=reader)
    assert m.wait_for_prefetch(3)
    rec = _buffer_record("random_ab/loading", m.loading_buffer, arrays)
    arrays["random_ab/filter_local"] = m.loading_buffer.filters_local[0].numpy().copy()
    rec["reader_calls"] = reader.calls
    meta["random_ab"] = rec
    arrays["random_ab/scene"] = scene.numpy()
    m.clear()

    # (3) persistent slots: full blocks, |incoming| == |evicted|, deferred copy.
    m = DB(num_total_gaussians=num_total, block_size=B, device="cpu", verbose=False)
    s = m.active_buffer
    active = [1, 2, 3, 4]
    rows = torch.cat([blocks[b] for b in active])
    for n, (a, b_) in cols.items():
        setattr(s, n, (rows[:, a:b_] + 1000.0).contiguous())
    s.local_to_global_idx = torch.cat([torch.arange(b * B, b * B + B) for b in active])
    s.loaded_blocks = list(active)
    s.block_to_local_slice = {b: slice(i * B, (i + 1) * B) for i, b in enumerate(active)}
    s.num_gaussians = len(active) * B
    reader = _Reader(br, br.BlockLayout.CACHE, blocks)
    m.start_prefetch(iteration=4, visible_block_ids=[2, 3, 5, 6], resident_block_ids=[2, 3],
                     evicted_block_ids=[1, 4], block_reader=reader, defer_resident_copy=True)
    h = m.finalize_retained_blocks([2, 3], target="loading")
    assert m.wait_for_prefetch(4)
    m.swap_buffers()
    rec = _buffer_record("persistent/active", m.active_buffer, arrays)
    st = m.get_stats()
    rec["stats"] = {k: st[k] for k in ("persistent_slot_updates", "persistent_omega_reuses",
                                       "persistent_streamed_blocks", "resident_refresh_blocks")}
    rec["handoff"] = [h.ready_blocks, h.copied_blocks]
    rec["reader_calls"] = reader.calls
    meta["persistent"] = rec
    m.clear()

    np.savez_compressed(out_dir / "double_buffer.npz", **arrays)
    (out_dir / "double_buffer.json").write_text(json.dumps(meta, indent=1))


def writeback(wset, out_dir: Path) -> None:
    arrays, meta = {}, {}
    B, num_total = 32, 7 * 32 - 9  # block 6 is a 23-row tail
    ws = wset.GPUWorkingSet(num_total_gaussians=num_total, block_size=B, device="cpu")
    gen = torch.Generator().manual_seed(9)
    order = [5, 1, 6, 3, 0]
    lengths = {b: min(B, num_total - b * B) for b in order}
    rows = sum(lengths.values())
    comps = {n: torch.randn((rows, WIDTHS[n]), generator=gen) * 50 for n in COMPONENTS}
    ws.gpu_xyz, ws.gpu_scaling, ws.gpu_rotation = comps["xyz"], comps["scaling"], comps["rotation"]
    ws.gpu_opacity, ws.gpu_features_dc = comps["opacity"], comps["features_dc"]
    ws.gpu_features_rest = comps["features_rest"]
    off = 0
    for b in order:
        # block 1's slice is shorter than the block: the plan clamps to it
        n = lengths[b] if b != 1 else 20
        ws.block_to_gpu_slice[b] = slice(off, off + n)
        off += lengths[b]
    ws.loaded_blocks = list(order)
    for n in COMPONENTS:
        arrays[f"comp/{n}"] = comps[n].numpy().copy()
    ids = [6, 3, 3, 9, 1, 5]  # unsorted, duplicate, not resident
    pending = ws.stage_updated_blocks(ids)
    packed = pending.wait()
    meta["plans"] = [[int(b), int(n)] for b, n in pending.plans]
    arrays["packed"] = pending.packed_cpu.numpy().copy()
    meta["block_ids"] = pending.block_ids
    meta["slices"] = {str(b): [s.start, s.stop] for b, s in ws.block_to_gpu_slice.items()}
    meta["block_size"] = B
    meta["num_total"] = num_total
    bounds = ws.stage_block_bounds([0, 6, 1, 42, 5])
    bids, cpu_bounds = bounds.wait()
    meta["bounds_ids"] = bids
    arrays["bounds"] = cpu_bounds.numpy()
    meta["writeback_stats"] = {k: v for k, v in ws.writeback_stats.items()
                               if k not in ("pinned_staging_bytes", "pinned_staging")}
    assert set(packed) == {1, 3, 5, 6}
    np.savez_compressed(out_dir / "writeback.npz", **arrays)
    (out_dir / "writeback.json").write_text(json.dumps(meta, indent=1))


def dirty(dbuf, out_dir: Path) -> None:
    meta = {}
    m = dbuf.DoubleBufferGPUWorkingSet(num_total_gaussians=16, block_size=4, device="cpu",
                                       verbose=False)
    meta["unit"] = {"mark": m.mark_dirty_blocks([0, 1, 1]),
                    "for_eviction": m.dirty_blocks_for_eviction([1, 2])}
    m.mark_blocks_written_back([1])
    meta["unit"]["dirty"] = m.dirty_blocks()
    m.clear()
    rng = np.random.default_rng(11)
    nb = 1000
    m = dbuf.DoubleBufferGPUWorkingSet(num_total_gaussians=nb * 8 - 3, block_size=8,
                                       device="cpu", verbose=False)
    mark = rng.integers(-20, nb + 20, 400).tolist()
    evict = rng.integers(-5, nb + 5, 300).tolist()
    back = rng.integers(0, nb, 100).tolist()
    rec = {"num_blocks": nb, "mark_ids": mark, "evict_ids": evict, "back_ids": back}
    rec["mark"] = m.mark_dirty_blocks(mark)
    rec["for_eviction"] = m.dirty_blocks_for_eviction(evict)
    m.mark_blocks_written_back(back)
    rec["dirty"] = m.dirty_blocks()
    rec["stats"] = {k: m.get_stats()[k] for k in ("dirty_blocks_marked",
                                                   "dirty_blocks_written_back")}
    meta["random"] = rec
    m.clear()
    # global -> local on a random table (negative, out-of-range and absent ids)
    starts = torch.full((50,), -1, dtype=torch.long)
    present = rng.choice(50, 20, replace=False)
    starts[present] = torch.from_numpy(rng.integers(0, 10_000, 20))
    gids = torch.from_numpy(rng.integers(-100, 50 * 8 + 100, 500))
    meta["g2l"] = {"block_size": 8, "block_starts": starts.tolist(), "gids": gids.tolist(),
                   "out": dbuf._global_ids_to_local(gids, starts, 8).tolist()}
    (out_dir / "dirty.json").write_text(json.dumps(meta, indent=1))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="path to the TideGS source tree")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args(argv)
    out = Path(args.out)
    torch.set_num_threads(1)
    br, dbuf, wset, gro = load_reference(Path(args.reference))
    resident_adam(gro, out)
    double_buffer(br, dbuf, out)
    writeback(wset, out)
    dirty(dbuf, out)
    print("golden fixtures written to", out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
