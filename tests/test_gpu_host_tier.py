"""GPU: the host tier on the device path. The write-back DMA lands in fresh
page-locked cache entries (GPUWorkingSet.stage_updated_blocks(...,
host_cache=...)), bit-equal to the oracle's CACHE-layout pack; the
materializer DMAs blocks straight out of cache entries (CachedBlockReader)
and records its reads on them."""
import numpy as np
import pytest
import torch

from oracle import blocks as ob

pytestmark = pytest.mark.gpu

NAMES = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")


class _Store:
    """Block store stand-in: block b holds a seeded CACHE-layout block."""

    def __init__(self, block_size, num_total):
        self.block_size, self.num_total = block_size, num_total
        self.writes = []

    def rows(self, b):
        return min(self.block_size, self.num_total - b * self.block_size)

    def block(self, b):
        rng = np.random.default_rng(700 + b)
        return torch.from_numpy(rng.standard_normal((self.rows(b), 59)).astype(np.float32))

    def read_blocks(self, ids):
        return {int(b): self.block(int(b)) for b in ids}

    def write_patch(self, blocks):
        self.writes.append(sorted(blocks))
        return len(self.writes)


def _cache(store, capacity):
    from tidegs_b200 import PinnedBlockCache

    return PinnedBlockCache(store, max_ram_gb=1e6, block_size=store.block_size, verbose=False,
                            capacity_blocks=capacity)


def test_writeback_lands_in_cache_entries():
    from tidegs_b200 import GPUWorkingSet

    B, nblk = 4096, 9
    num_total = B * nblk - 1000  # the last block is short
    gen = torch.Generator(device="cuda").manual_seed(5)
    comps = {n: torch.randn((nblk * B, w), generator=gen, device="cuda")
             for n, w in ob.WIDTHS.items()}
    ws = GPUWorkingSet(num_total_gaussians=num_total, block_size=B, device="cuda")
    ws.gpu_xyz, ws.gpu_scaling, ws.gpu_rotation = comps["xyz"], comps["scaling"], comps["rotation"]
    ws.gpu_opacity, ws.gpu_features_dc = comps["opacity"], comps["features_dc"]
    ws.gpu_features_rest = comps["features_rest"]
    order = [4, 8, 0, 2, 6, 1, 7, 3, 5]  # block in slot i
    for i, b in enumerate(order):
        ws.block_to_gpu_slice[b] = slice(i * B, (i + 1) * B)
    store = _Store(B, num_total)
    cache = _cache(store, 16)
    host = {n: comps[n].cpu().numpy() for n in NAMES}
    try:
        assert cache.slab.is_pinned()
        for rnd, ids in enumerate(([8, 3, 6, 0], [6, 8, 1])):
            if rnd == 1:
                for t in comps.values():
                    t.mul_(-0.5)
                host = {n: comps[n].cpu().numpy() for n in NAMES}
            free_before = cache.get_stats()["free_entries"]
            pending = ws.stage_updated_blocks(ids, host_cache=cache)
            assert pending.packed_cpu is None
            result = pending.wait()
            assert sorted(result) == sorted(ids) == pending.block_ids
            for b in ids:
                slot = order.index(b)
                want = ob.pack_rows(host, [slot * B], [store.rows(b)], "cache")
                np.testing.assert_array_equal(result[b].numpy(), want)
                assert torch.equal(cache.cache_data[b], result[b])
                assert cache.block_versions[b] == (2 if rnd == 1 and b in (8, 6) else 1)
            assert cache.dirty_set >= set(ids)
            # rewritten blocks free their previous entries
            reused = len(set(ids) & {8, 3, 6, 0}) if rnd == 1 else 0
            assert cache.get_stats()["free_entries"] == free_before - len(ids) + reused
            pending.release()
        assert ws.writeback_stats["direct_cache_d2h_blocks"] == 7
        assert cache.get_stats()["direct_writeback_blocks"] == 7
        cache.flush_all_dirty()
        assert store.writes == [[0, 1, 3, 6, 8]]
    finally:
        cache.shutdown()


def test_materializer_dmas_from_cache_entries():
    from tidegs_b200 import CachedBlockReader, DoubleBufferGPUWorkingSet

    B, nblk = 2048, 12
    num_total = B * nblk
    store = _Store(B, num_total)
    cache = _cache(store, 32)
    reader = CachedBlockReader(cache, num_total, B)
    manager = DoubleBufferGPUWorkingSet(num_total, B, device="cuda", verbose=False)
    try:
        visible = [9, 2, 5, 11, 0]
        manager.start_prefetch(iteration=3, visible_block_ids=visible, block_reader=reader)
        assert manager.wait_for_prefetch(3)
        manager.swap_buffers()
        act = manager.active_buffer
        assert act.loaded_blocks == sorted(visible)
        packed = torch.cat([store.block(b) for b in sorted(visible)]).numpy()
        cols = ob.columns("cache")
        for n, w in ob.WIDTHS.items():
            np.testing.assert_array_equal(getattr(act, n).cpu().numpy(),
                                          packed[:, cols[n]:cols[n] + w])
        gids = np.concatenate([np.arange(b * B, (b + 1) * B) for b in sorted(visible)])
        np.testing.assert_array_equal(act.local_to_global_idx.cpu().numpy(), gids)
        stats = cache.get_stats()
        assert stats["cache_misses"] == len(visible)  # read from the store into entries
        with cache.cache_lock:
            noted = {cache._entry_of(cache.cache_data[b]) for b in visible}
            assert noted <= set(cache._dma_reads)
        # a second prefetch of the same blocks hits the cache
        manager.start_prefetch(iteration=4, visible_block_ids=visible, block_reader=reader)
        assert manager.wait_for_prefetch(4)
        assert cache.get_stats()["cache_hits"] == len(visible)
    finally:
        manager.clear()
        cache.shutdown()
