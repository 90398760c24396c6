"""GPU parity of DoubleBufferGPUWorkingSet: the reference's
tests/test_double_buffer_materialization.py ported to this package, plus
bit-exact comparisons with golden outputs of the reference's own CPU run."""
import threading
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")


def _components(global_ids):
    rows = global_ids.to(dtype=torch.float32).unsqueeze(1)
    return {
        "xyz": rows + torch.tensor([0.1, 0.2, 0.3], device=rows.device),
        "scaling": rows + torch.tensor([1.1, 1.2, 1.3], device=rows.device),
        "rotation": rows + torch.tensor([2.1, 2.2, 2.3, 2.4], device=rows.device),
        "opacity": rows + 3.1,
        "features_dc": rows + torch.tensor([4.1, 4.2, 4.3], device=rows.device),
        "features_rest": rows + torch.arange(45, device=rows.device) * 0.01 + 5.0,
    }


def _pack_block(global_ids, layout):
    from tidegs_b200.block_reader import BlockLayout

    values = _components(global_ids)
    if layout == BlockLayout.CACHE:
        order = ("xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest")
    else:
        order = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")
    return torch.cat([values[name] for name in order], dim=1).cpu()


class _Reader:
    def __init__(self, layout, blocks):
        self.layout = layout
        self.blocks = blocks
        self.calls = []

    def read_blocks(self, block_ids):
        self.calls.append(list(block_ids))
        return {block_id: self.blocks[block_id] for block_id in block_ids}

    def read_batch(self, block_ids, out=None):
        from tidegs_b200.block_reader import _pack_block_batch

        return _pack_block_batch(self.read_blocks(block_ids), block_ids, self.layout, out)


class _BlockingReader(_Reader):
    def __init__(self, layout, blocks):
        super().__init__(layout, blocks)
        self.started = threading.Event()
        self.release = threading.Event()

    def read_blocks(self, block_ids):
        self.started.set()
        if not self.release.wait(timeout=2.0):
            raise TimeoutError("test did not release the blocking reader")
        return super().read_blocks(block_ids)


def _manager(num_total, block_size):
    from tidegs_b200 import DoubleBufferGPUWorkingSet

    return DoubleBufferGPUWorkingSet(num_total_gaussians=num_total, block_size=block_size,
                                     device="cuda", verbose=False)


def test_reused_staging_slot_exposes_only_requested_rows():
    manager = _manager(32, 4)
    try:
        first_cpu, first_gpu, first_slot = manager._acquire_host_staging(8)
        manager._acquire_host_staging(4)
        reused_cpu, reused_gpu, reused_slot = manager._acquire_host_staging(3)
        assert first_slot == reused_slot
        assert tuple(reused_cpu.shape) == (3, 59)
        assert tuple(reused_gpu.shape) == (3, 59)
        assert first_cpu.data_ptr() == reused_cpu.data_ptr()
        assert first_gpu.data_ptr() == reused_gpu.data_ptr()
    finally:
        manager.clear()


@pytest.mark.parametrize("layout_name", ["cache", "unified"])
def test_layouts_match_reference_test_and_golden(golden, layout_name):
    from tidegs_b200.block_reader import BlockLayout

    layout = BlockLayout.CACHE if layout_name == "cache" else BlockLayout.UNIFIED
    meta, arrays = golden("double_buffer")
    rec = meta[f"unit_{layout_name}"]
    manager = _manager(14, 4)
    try:
        source_ids = torch.tensor([4, 5, 6, 7, 12, 13], device="cuda")
        source_values = _components(source_ids)
        source = manager.active_buffer
        for name in NAMES:
            setattr(source, name, source_values[name])
        source.local_to_global_idx = source_ids
        source.loaded_blocks = [1, 3]
        source.block_to_local_slice = {1: slice(0, 4), 3: slice(4, 6)}
        source.num_gaussians = 6
        reader = _Reader(layout, {2: _pack_block(torch.tensor([8, 9, 10, 11]), layout)})
        manager.start_prefetch(iteration=17, visible_block_ids=[3, 2, 1],
                               resident_block_ids=[1, 3], evicted_block_ids=[0],
                               block_reader=reader)
        assert manager.wait_for_prefetch(17)
        target = manager.loading_buffer
        expected_ids = torch.tensor([4, 5, 6, 7, 12, 13, 8, 9, 10, 11], device="cuda")
        expected = _components(expected_ids)
        torch.testing.assert_close(target.local_to_global_idx, expected_ids)
        for name, exp in expected.items():
            torch.testing.assert_close(getattr(target, name), exp, rtol=0, atol=0)
            np.testing.assert_array_equal(getattr(target, name).cpu().numpy(),
                                          arrays[f"unit_{layout_name}/loading/{name}"])
        assert target.loaded_blocks == rec["loaded_blocks"] == [1, 3, 2]
        assert target.resident_blocks == [1, 3]
        assert target.streamed_blocks == [2]
        assert target.evicted_blocks == [0]
        assert reader.calls == [[2]]
        assert target.block_to_local_slice[1] == slice(0, 4)
        assert target.block_to_local_slice[3] == slice(4, 6)
        assert target.block_to_local_slice[2] == slice(6, 10)
        assert target._block_starts[[1, 2, 3]].cpu().tolist() == [0, 6, 4]
        np.testing.assert_array_equal(target._block_starts.cpu().numpy(),
                                      arrays[f"unit_{layout_name}/loading/block_starts"])
        stats = manager.get_stats()
        for k, v in rec["stats"].items():
            assert stats[k] == v, k
        for name in expected:
            getattr(source, name).add_(10.0)
        handoff = manager.finalize_retained_blocks([1, 3], target="loading")
        assert [handoff.ready_blocks, handoff.copied_blocks] == rec["handoff"]
        manager.prefetch_complete_event.synchronize()
        torch.cuda.synchronize()
        for name in expected:
            np.testing.assert_array_equal(getattr(target, name).cpu().numpy(),
                                          arrays[f"unit_{layout_name}/refreshed/{name}"])
        manager.swap_buffers()
        query = torch.tensor([4, 12, 8], device="cuda")
        assert manager.global_to_local(query).cpu().tolist() == rec["global_to_local_4_12_8"]
    finally:
        manager.clear()


def test_dirty_blocks_are_written_back_only_on_eviction(golden):
    meta, _ = golden("dirty")
    manager = _manager(16, 4)
    try:
        assert manager.mark_dirty_blocks([0, 1, 1]) == meta["unit"]["mark"] == 2
        assert manager.dirty_blocks_for_eviction([1, 2]) == meta["unit"]["for_eviction"] == [1]
        manager.mark_blocks_written_back([1])
        assert manager.dirty_blocks() == meta["unit"]["dirty"] == [0]
    finally:
        manager.clear()


def test_dirty_bitmap_random_matches_golden(golden):
    meta, _ = golden("dirty")
    rec = meta["random"]
    manager = _manager(rec["num_blocks"] * 8 - 3, 8)
    try:
        assert manager.mark_dirty_blocks(rec["mark_ids"]) == rec["mark"]
        assert manager.dirty_blocks_for_eviction(rec["evict_ids"]) == rec["for_eviction"]
        manager.mark_blocks_written_back(rec["back_ids"])
        assert manager.dirty_blocks() == rec["dirty"]
        st = manager.get_stats()
        for k, v in rec["stats"].items():
            assert st[k] == v
    finally:
        manager.clear()


def test_resident_plan_runs_on_background_worker():
    manager = _manager(16, 4)
    try:
        started = threading.Event()
        release = threading.Event()

        def planner():
            started.set()
            if not release.wait(timeout=2.0):
                raise TimeoutError("resident planner test was not released")
            return {"planned": True}

        future = manager.submit_resident_plan(17, planner)
        assert started.wait(timeout=1.0)
        assert not future.done()
        release.set()
        assert future.result(timeout=2.0) == {"planned": True}
        assert manager.get_stats()["resident_plan_jobs"] == 1
    finally:
        manager.clear()


def test_persistent_slots_keep_omega_and_fill_only_delta():
    from tidegs_b200.block_reader import BlockLayout

    manager = _manager(16, 4)
    try:
        source_ids = torch.tensor([0, 1, 2, 3, 4, 5, 6, 7], device="cuda")
        source_values = _components(source_ids)
        source = manager.active_buffer
        for name, tensor in source_values.items():
            setattr(source, name, tensor)
        source.local_to_global_idx = source_ids.clone()
        source.loaded_blocks = [0, 1]
        source.block_to_local_slice = {0: slice(0, 4), 1: slice(4, 8)}
        source.num_gaussians = 8
        reader = _Reader(BlockLayout.CACHE,
                         {2: _pack_block(torch.tensor([8, 9, 10, 11]), BlockLayout.CACHE)})
        fences = []
        manager.start_prefetch(iteration=17, visible_block_ids=[1, 2], resident_block_ids=[1],
                               evicted_block_ids=[0], block_reader=reader,
                               defer_resident_copy=True,
                               before_target_reuse=lambda: fences.append("activation"))
        for name in source_values:
            getattr(source, name)[4:8].add_(10.0)
        original = manager._copy_resident_blocks

        def _fail(*a, **k):
            raise AssertionError("persistent Omega handoff must not copy resident tensors")

        manager._copy_resident_blocks = _fail
        try:
            handoff = manager.finalize_retained_blocks([1], target="loading")
        finally:
            manager._copy_resident_blocks = original
        assert handoff.ready_blocks == 1 and handoff.copied_blocks == 0
        assert manager.wait_for_prefetch(17)
        assert fences == []
        manager.swap_buffers()
        assert fences == ["activation"]
        assert manager.active_buffer is source
        assert manager.active_buffer.loaded_blocks == [2, 1]
        assert manager.active_buffer.block_to_local_slice[2] == slice(0, 4)
        assert manager.active_buffer.block_to_local_slice[1] == slice(4, 8)
        assert reader.calls == [[2]]
        expected_ids = torch.tensor([8, 9, 10, 11, 4, 5, 6, 7], device="cuda")
        expected = _components(expected_ids)
        for name in expected:
            expected[name][4:8].add_(10.0)
            torch.testing.assert_close(getattr(source, name), expected[name], rtol=0, atol=0)
        torch.testing.assert_close(source.local_to_global_idx, expected_ids)
        stats = manager.get_stats()
        assert stats["persistent_slot_updates"] == 1
        assert stats["persistent_omega_reuses"] == 1
        assert stats["resident_refresh_blocks"] == 0
    finally:
        manager.clear()


def test_block_reader_prefetch_returns_before_read_and_defers_resident_copy():
    from tidegs_b200.block_reader import BlockLayout

    manager = _manager(12, 4)
    try:
        source_ids = torch.tensor([0, 1, 2, 3], device="cuda")
        source_values = _components(source_ids)
        source = manager.active_buffer
        for name, tensor in source_values.items():
            setattr(source, name, tensor)
        source.local_to_global_idx = source_ids
        source.loaded_blocks = [0]
        source.block_to_local_slice = {0: slice(0, 4)}
        source.num_gaussians = 4
        reader = _BlockingReader(BlockLayout.CACHE,
                                 {1: _pack_block(torch.tensor([4, 5, 6, 7]), BlockLayout.CACHE)})
        started_at = time.perf_counter()
        manager.start_prefetch(iteration=17, visible_block_ids=[0, 1], resident_block_ids=[0],
                               block_reader=reader, defer_resident_copy=True)
        assert time.perf_counter() - started_at < 0.5
        assert reader.started.wait(timeout=1.0)
        for name in source_values:
            getattr(source, name).add_(10.0)
        refresh_started = time.perf_counter()
        try:
            handoff = manager.finalize_retained_blocks([0], target="loading")
            assert handoff.ready_blocks == 1 and handoff.copied_blocks == 1
            assert time.perf_counter() - refresh_started < 1.5
            assert not reader.release.is_set()
        finally:
            reader.release.set()
        assert manager.wait_for_prefetch(17)
        target = manager.loading_buffer
        expected = _components(torch.tensor([0, 1, 2, 3, 4, 5, 6, 7], device="cuda"))
        for name in expected:
            expected[name][:4].add_(10.0)
            torch.testing.assert_close(getattr(target, name), expected[name], rtol=0, atol=0)
    finally:
        manager.clear()


def _seed_active(manager, blocks, active, B, num_total):
    s = manager.active_buffer
    rows = torch.cat([blocks[b] for b in active])
    cols = {"xyz": (0, 3), "scaling": (3, 6), "rotation": (6, 10), "opacity": (10, 11),
            "features_dc": (11, 14), "features_rest": (14, 59)}
    for n, (a, b_) in cols.items():
        setattr(s, n, (rows[:, a:b_] + 1000.0).contiguous().cuda())
    s.local_to_global_idx = torch.cat([torch.arange(b * B, b * B + B) for b in active]).cuda()
    s.loaded_blocks = list(active)
    s.block_to_local_slice = {b: slice(i * B, (i + 1) * B) for i, b in enumerate(active)}
    s.num_gaussians = len(active) * B


def _check_buffer(buf, rec, arrays, prefix):
    for n in NAMES:
        np.testing.assert_array_equal(getattr(buf, n).cpu().numpy(), arrays[f"{prefix}/{n}"],
                                      err_msg=n)
    np.testing.assert_array_equal(buf.local_to_global_idx.cpu().numpy(), arrays[f"{prefix}/gids"])
    np.testing.assert_array_equal(buf._block_starts.cpu().numpy(),
                                  arrays[f"{prefix}/block_starts"])
    assert buf.loaded_blocks == rec["loaded_blocks"]
    assert buf.resident_blocks == rec["resident_blocks"]
    assert buf.streamed_blocks == rec["streamed_blocks"]
    assert buf.evicted_blocks == rec["evicted_blocks"]
    assert {str(b): [s.start, s.stop] for b, s in buf.block_to_local_slice.items()} == rec["slices"]


class _PinnedViews:
    """A reader exposing only page-locked per-block views."""

    def __init__(self, pool):
        self._pool = pool
        self.layout = pool.layout

    def read_blocks_pinned(self, ids):
        return self._pool.read_blocks_pinned(ids)


@pytest.mark.parametrize("source", ["read_batch", "pool_pointers", "pinned_views"])
def test_random_ab_materialization_matches_golden(golden, source):
    from tidegs_b200.block_reader import BlockLayout, PinnedBlockPool

    meta, arrays = golden("double_buffer")
    rec = meta["random_ab"]
    B, nblocks, tail = 16, 20, 11
    num_total = (nblocks - 1) * B + tail
    scene = torch.from_numpy(arrays["random_ab/scene"])
    blocks = {b: scene[b * B: min((b + 1) * B, num_total)].clone() for b in range(nblocks)}
    manager = _manager(num_total, B)
    try:
        _seed_active(manager, blocks, [0, 2, 4, 6], B, num_total)
        pinned_pool = source != "read_batch"
        if pinned_pool:
            pool = torch.zeros((nblocks, B, 59))
            for b, rows in blocks.items():
                pool[b, : rows.shape[0]] = rows
            reader = PinnedBlockPool(pool, B, num_total, layout=BlockLayout.CACHE)
            if source == "pinned_views":
                reader = _PinnedViews(reader)
        else:
            reader = _Reader(BlockLayout.CACHE, blocks)
        filt = torch.tensor([2 * B + 3, 7 * B, 5 * B + 1, 19 * B + 10, 19 * B + 12, -5, 4 * B + 15])
        manager.start_prefetch(iteration=3, visible_block_ids=[7, 4, 2, 19, 3],
                               filters_global=[filt], resident_block_ids=[2, 4],
                               evicted_block_ids=[0, 6], block_reader=reader)
        assert manager.wait_for_prefetch(3)
        _check_buffer(manager.loading_buffer, rec, arrays, "random_ab/loading")
        np.testing.assert_array_equal(manager.loading_buffer.filters_local[0].cpu().numpy(),
                                      arrays["random_ab/filter_local"])
        if pinned_pool:
            assert manager.get_stats()["direct_block_dma_calls"] == 3
        else:
            assert reader.calls == rec["reader_calls"]
    finally:
        manager.clear()


def test_persistent_plan_matches_golden(golden):
    from tidegs_b200.block_reader import BlockLayout

    meta, arrays = golden("double_buffer")
    rec = meta["persistent"]
    B, nblocks, tail = 16, 20, 11
    num_total = (nblocks - 1) * B + tail
    scene = torch.from_numpy(arrays["random_ab/scene"])
    blocks = {b: scene[b * B: min((b + 1) * B, num_total)].clone() for b in range(nblocks)}
    manager = _manager(num_total, B)
    try:
        _seed_active(manager, blocks, [1, 2, 3, 4], B, num_total)
        reader = _Reader(BlockLayout.CACHE, blocks)
        manager.start_prefetch(iteration=4, visible_block_ids=[2, 3, 5, 6],
                               resident_block_ids=[2, 3], evicted_block_ids=[1, 4],
                               block_reader=reader, defer_resident_copy=True)
        h = manager.finalize_retained_blocks([2, 3], target="loading")
        assert [h.ready_blocks, h.copied_blocks] == rec["handoff"]
        assert manager.wait_for_prefetch(4)
        manager.swap_buffers()
        torch.cuda.synchronize()
        _check_buffer(manager.active_buffer, rec, arrays, "persistent/active")
        st = manager.get_stats()
        for k, v in rec["stats"].items():
            assert st[k] == v, k
        assert reader.calls == rec["reader_calls"]
    finally:
        manager.clear()
