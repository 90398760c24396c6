"""CPU: the host tier (tidegs_b200/host_tier.py) against the reference.

* BlockLogStore replays the reference LogStorageManager's patch sequence of
  tests/golden/host_tier.json: identical patch bytes (sha256), index
  (file, offset, size, version), read order and contents, statistics and
  error messages.
* PinnedBlockCache replays three seeded 60-operation sequences recorded on
  the reference TieredCacheManager (upserts, prefetches with misses,
  dirty submissions with and without clone, future prefetch, eviction,
  flush_all): after every operation the LRU order, contents, dirty set,
  versions, flushing buffer, statistics and the store's write log match.
* The reference's single-flight tests (tests/test_tiered_cache_singleflight.py)
  ported to PinnedBlockCache, plus slab-entry accounting and a cache + block
  log round trip.
"""
import hashlib
import json
import sys
import threading
import time
from pathlib import Path

import numpy as np
import pytest
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_host_tier_golden as G  # noqa: E402

from tidegs_b200.host_tier import BlockLogStore, CachedBlockReader, PinnedBlockCache  # noqa: E402

FIX = json.loads((HERE / "golden" / "host_tier.json").read_text())


def _cache(store, max_ram_gb, block_size, capacity=64):
    return PinnedBlockCache(store, max_ram_gb=max_ram_gb, block_size=block_size,
                            point_dim=G.POINT_DIM, verbose=False, capacity_blocks=capacity,
                            pin_memory=False)


def _assert_entries_consistent(cache):
    """Every slab entry is free or referenced; cache views are slab entries."""
    with cache.cache_lock:
        held = int((cache._refs > 0).sum())
        assert held + len(cache._free) == cache.capacity_blocks
        assert len(set(cache._free)) == len(cache._free)
        for b, v in cache.cache_data.items():
            assert cache._entry_of(v) == cache._cache_entry[b]
            assert cache._refs[cache._cache_entry[b]] >= 1


def test_block_log_matches_reference_patches(tmp_path):
    ref = FIX["log"]
    B, NB = ref["block_size"], ref["num_blocks"]
    st = BlockLogStore(str(tmp_path), B, NB, point_dim=G.POINT_DIM, verbose=False)
    base = torch.cat([G.block_data(20_000 + b, B) for b in range(NB)])
    st.file_paths[0].write_bytes(base.numpy().tobytes())
    for p in ref["patches"]:
        blocks = {int(b): (G.block_data(30_000 + s, r) if r else torch.empty((0, G.POINT_DIM)))
                  for b, (r, s) in p["spec"].items()}
        pid = st.write_patch(blocks)
        assert pid == p["patch_id"]
        path = st.file_paths[pid]
        assert hashlib.sha256(path.read_bytes()).hexdigest() == p["sha256"]
        assert path.stat().st_size == p["size"]
        index = {str(b): [l.file_id, l.offset, l.size, l.version] for b, l in sorted(st.index.items())}
        assert index == p["index"]
    got = st.read_blocks([5, 0, 3, 1, 2, 4])
    assert [int(b) for b in got] == ref["read_order"]
    assert {str(b): [list(t.shape), G.digest(t)] for b, t in got.items()} == ref["read"]
    s = st.get_stats()
    assert {k: int(s[k]) for k in ref["stats"]} == ref["stats"]
    with pytest.raises(ValueError) as e:
        st.write_patch({0: torch.zeros((2, 3))})
    assert str(e.value) == ref["errors"]["bad_width"]
    with pytest.raises(ValueError) as e:
        st.write_patch({0: torch.zeros((B + 1, G.POINT_DIM))})
    assert str(e.value) == ref["errors"]["too_many_rows"]
    with pytest.raises(ValueError) as e:
        st.read_blocks([NB + 3])
    assert str(e.value) == ref["errors"]["missing"]
    # zero-copy reads into caller memory equal the plain reads
    dest = {b: torch.full((B, G.POINT_DIM), -1.0) for b in range(NB)}
    rows = st.read_blocks_into(list(range(NB)), dest)
    for b in range(NB):
        assert torch.equal(dest[b][:rows[b]], got[b])
    assert list(rows) == [int(b) for b in st.read_blocks(list(range(NB)))]
    st.close()


@pytest.mark.parametrize("k", [0, 1, 2])
def test_cache_sequence_matches_reference(k):
    ref = FIX["cache"][k]
    B = ref["block_size"]
    store = G.RecordingStore(B)
    cache = _cache(store, ref["max_ram_gb"], B)
    try:
        for i, (op, want) in enumerate(zip(ref["ops"], ref["steps"])):
            result = G.apply_cache_op(cache, op, B)
            got = {"result": result, **G.cache_state(cache, store)}
            assert got == want, f"seed {ref['seed']} step {i} op {op}"
            _assert_entries_consistent(cache)
    finally:
        cache.shutdown()
    # the write log includes the dirty blocks shutdown() flushed
    assert store.writes == ref["writes"]
    with cache.cache_lock:
        assert not cache.flushing_buffer and not cache.dirty_set
        assert int(cache._refs.sum()) == len(cache.cache_data)


class _FakeStorage:
    """Port of the reference test's FakeStorage (blocking / failing first read)."""

    def __init__(self, block_size=2, point_dim=G.POINT_DIM):
        self.block_size, self.point_dim = block_size, point_dim
        self.data = {b: torch.full((block_size, point_dim), float(b)) for b in range(32)}
        self.read_counts = {}
        self.call_count = 0
        self.lock = threading.Lock()
        self.block_first_read = False
        self.fail_first_read = False
        self.read_started = threading.Event()
        self.release_read = threading.Event()

    def read_blocks(self, block_ids):
        block_ids = [int(b) for b in block_ids]
        with self.lock:
            self.call_count += 1
            call = self.call_count
            for b in block_ids:
                self.read_counts[b] = self.read_counts.get(b, 0) + 1
        if self.block_first_read and call == 1:
            self.read_started.set()
            if not self.release_read.wait(timeout=2.0):
                raise TimeoutError("test timed out waiting to release first read")
        if self.fail_first_read and call == 1:
            raise RuntimeError("injected read failure")
        return {b: self.data[b].clone() for b in block_ids}

    def write_patch(self, blocks):
        return None


def _small_cache(storage):
    return PinnedBlockCache(storage, max_ram_gb=1.0, block_size=storage.block_size,
                            point_dim=storage.point_dim, verbose=False, capacity_blocks=64,
                            pin_memory=False)


def _prefetch_in_thread(cache, ids):
    result, errors = {}, []

    def target():
        try:
            result.update(cache.prefetch(ids))
        except Exception as exc:  # asserted by the tests
            errors.append(exc)

    t = threading.Thread(target=target)
    t.start()
    return t, result, errors


def test_dirty_batch_views_share_one_slab():
    storage = _FakeStorage()
    cache = _small_cache(storage)
    try:
        source = torch.arange(2 * 2 * G.POINT_DIM, dtype=torch.float32).reshape(4, G.POINT_DIM)
        expected = source.clone()
        assert cache.upsert_dirty_block_batch({5: source[:2], 6: source[2:]}) == 2
        source.add_(100.0)
        assert torch.equal(cache.cache_data[5], expected[:2])
        assert torch.equal(cache.cache_data[6], expected[2:])
        assert (cache.cache_data[5].untyped_storage().data_ptr()
                == cache.cache_data[6].untyped_storage().data_ptr())
        assert cache.dirty_set == {5, 6}
    finally:
        cache.shutdown()


def test_future_read_serves_urgent_without_second_read():
    storage = _FakeStorage()
    storage.block_first_read = True
    cache = _small_cache(storage)
    try:
        assert cache.prefetch_future([7]) == 1
        assert storage.read_started.wait(timeout=2.0)
        t, result, errors = _prefetch_in_thread(cache, [7])
        time.sleep(0.05)
        assert t.is_alive()
        storage.release_read.set()
        t.join(timeout=2.0)
        assert not t.is_alive() and errors == []
        assert torch.equal(result[7], storage.data[7])
        assert storage.read_counts[7] == 1
        stats = cache.get_stats()
        assert stats["urgent_prefetch_blocks"] == 0
        assert stats["future_prefetch_reserved"] == 1
        assert stats["inflight_wait_blocks"] >= 1
    finally:
        cache.shutdown()


def test_future_hint_skips_block_claimed_by_urgent():
    storage = _FakeStorage()
    storage.block_first_read = True
    cache = _small_cache(storage)
    try:
        t, result, errors = _prefetch_in_thread(cache, [3])
        assert storage.read_started.wait(timeout=2.0)
        assert cache.prefetch_future([3]) == 0
        storage.release_read.set()
        t.join(timeout=2.0)
        assert not t.is_alive() and errors == []
        assert torch.equal(result[3], storage.data[3])
        assert storage.read_counts[3] == 1
        assert cache.get_stats()["future_prefetch_skipped"] >= 1
    finally:
        cache.shutdown()


def test_two_urgent_prefetches_share_one_read():
    storage = _FakeStorage()
    storage.block_first_read = True
    cache = _small_cache(storage)
    try:
        ta, ra, ea = _prefetch_in_thread(cache, [5])
        assert storage.read_started.wait(timeout=2.0)
        tb, rb, eb = _prefetch_in_thread(cache, [5])
        time.sleep(0.05)
        assert tb.is_alive()
        storage.release_read.set()
        ta.join(timeout=2.0)
        tb.join(timeout=2.0)
        assert not ta.is_alive() and not tb.is_alive() and ea == [] and eb == []
        assert torch.equal(ra[5], storage.data[5]) and torch.equal(rb[5], storage.data[5])
        assert storage.read_counts[5] == 1
        assert cache.get_stats()["urgent_prefetch_blocks"] == 1
    finally:
        cache.shutdown()


def test_flushing_buffer_hit_touches_no_storage():
    storage = _FakeStorage()
    cache = _small_cache(storage)
    try:
        assert cache.upsert_dirty_blocks({9: torch.full((2, G.POINT_DIM), 9.0)}) == 1
        tensor = cache.cache_data[9]
        with cache.flushing_lock:
            cache.flushing_buffer[9] = (tensor, time.time(), 0)
        with cache.cache_lock:
            cache.cache_data.pop(9)
        result = cache.prefetch([9])
        assert torch.equal(result[9], torch.full((2, G.POINT_DIM), 9.0))
        assert storage.read_counts.get(9, 0) == 0
        assert cache.get_stats()["inflight_read_blocks"] == 0
        with cache.flushing_lock:
            cache.flushing_buffer.pop(9, None)
    finally:
        cache.shutdown()


def test_future_failure_wakes_urgent_and_falls_back():
    storage = _FakeStorage()
    storage.block_first_read = True
    storage.fail_first_read = True
    cache = _small_cache(storage)
    try:
        assert cache.prefetch_future([11]) == 1
        assert storage.read_started.wait(timeout=2.0)
        t, result, errors = _prefetch_in_thread(cache, [11])
        time.sleep(0.05)
        assert t.is_alive()
        storage.release_read.set()
        t.join(timeout=2.0)
        assert not t.is_alive() and errors == []
        assert torch.equal(result[11], storage.data[11])
        assert storage.read_counts[11] == 2
        stats = cache.get_stats()
        assert stats["future_prefetch_errors"] == 1
        assert stats["inflight_fallback_blocks"] >= 1
    finally:
        cache.shutdown()


def test_cache_over_block_log_round_trip(tmp_path):
    """Dirty blocks evicted from a small cache reach the block log as patches
    and come back bit for bit; reserve/commit write-back publishes entries."""
    B, NB = 8, 40
    st = BlockLogStore(str(tmp_path), B, NB, point_dim=G.POINT_DIM, verbose=False)
    base = torch.cat([G.block_data(40_000 + b, B) for b in range(NB)])
    st.file_paths[0].write_bytes(base.numpy().tobytes())
    max_blocks = 6
    cache = PinnedBlockCache(st, max_ram_gb=max_blocks * B * G.POINT_DIM * 4 / 1024 ** 3,
                             block_size=B, point_dim=G.POINT_DIM, verbose=False,
                             capacity_blocks=24, pin_memory=False)
    want = {b: G.block_data(40_000 + b, B) for b in range(NB)}
    try:
        rng = np.random.default_rng(0)
        for step in range(30):
            ids = sorted(rng.choice(NB, 3, replace=False).tolist())
            plans = [(b, B) for b in ids]
            views = cache.reserve_writeback(plans)
            for (b, _), v in zip(plans, views):
                want[b] = G.block_data(50_000 + 100 * step + b, B)
                v.copy_(want[b])
            assert cache.commit_writeback(plans, views) == 3
            got = cache.prefetch(rng.choice(NB, 4, replace=False).tolist())
            for b, t in got.items():
                assert torch.equal(t, want[b]), (step, b)
            _assert_entries_consistent(cache)
        cache.drain()
        cache.flush_all_dirty()
        assert st.get_stats()["patches_created"] > 0
        fresh = st.read_blocks(list(range(NB)))
        for b in range(NB):
            assert torch.equal(fresh[b], want[b]), b
        reader = CachedBlockReader(cache, NB * B, B)
        ptrs, rows = reader.block_host_pointers([3, 17])
        assert rows.tolist() == [B, B]
        assert ptrs[0] == cache.cache_data[3].data_ptr()
        with pytest.raises(KeyError):
            reader.block_host_pointers([NB])
        batch = reader.read_batch([4, 2])
        assert torch.equal(batch.tensor, torch.cat([want[4], want[2]]))
    finally:
        cache.shutdown()
        st.close()


def test_tail_block_round_trip(tmp_path):
    """A scene whose last block is short (total rows not a multiple of the
    block size): its write-back entry holds only its rows, the patch stores
    only those rows, and the block comes back with that shape from the cache
    and from the log; the reader packs it with its real row count."""
    B, NB, tail = 8, 5, 3
    st = BlockLogStore(str(tmp_path), B, NB, point_dim=G.POINT_DIM, verbose=False)
    base = torch.cat([G.block_data(60_000 + b, B) for b in range(NB)])
    st.file_paths[0].write_bytes(base.numpy().tobytes())
    cache = PinnedBlockCache(st, max_ram_gb=1.0, block_size=B, point_dim=G.POINT_DIM,
                             verbose=False, capacity_blocks=8, pin_memory=False)
    try:
        plans = [(1, B), (NB - 1, tail)]
        views = cache.reserve_writeback(plans)
        new = {b: G.block_data(70_000 + b, rows) for b, rows in plans}
        for (b, _), v in zip(plans, views):
            assert v.shape == new[b].shape
            v.copy_(new[b])
        cache.commit_writeback(plans, views)
        got = cache.prefetch([NB - 1, 1])
        assert torch.equal(got[NB - 1], new[NB - 1]) and torch.equal(got[1], new[1])
        with pytest.raises(ValueError, match="rows"):
            cache.reserve_writeback([(2, B + 1)])
        cache.flush_all_dirty()
        cache.drain()
        assert st.index[NB - 1].size == tail * G.POINT_DIM * 4
        back = st.read_blocks([NB - 1, 1, 0])
        assert torch.equal(back[NB - 1], new[NB - 1]) and torch.equal(back[1], new[1])
        assert torch.equal(back[0], base[:B])
        reader = CachedBlockReader(cache, (NB - 1) * B + tail, B)
        batch = reader.read_batch([NB - 1, 1])
        assert torch.equal(batch.tensor, torch.cat([new[NB - 1], new[1]]))
    finally:
        cache.shutdown()
        st.close()



class _GatedLog(BlockLogStore):
    """Block log whose first write waits for `gate` (a slow disk)."""

    def __init__(self, *a, **k):
        super().__init__(*a, **k)
        self.gate = threading.Event()
        self.first = True

    def write_patch(self, block_dict):
        if self.first:
            self.first = False
            assert self.gate.wait(10.0)
        return super().write_patch(block_dict)


def test_synchronous_fallback_write_waits_for_queued_older_versions(tmp_path):
    """Flush queue full: the synchronous write of a block's newest version
    must land after the queued writes of its older versions, or the block
    log would keep an older one."""
    from queue import Queue

    B, NB = 8, 4
    st = _GatedLog(str(tmp_path), B, NB, point_dim=G.POINT_DIM, verbose=False)
    cache = _cache(st, max_ram_gb=1.0, block_size=B, capacity=16)
    cache.flush_queue = Queue(maxsize=1)
    try:
        versions = [G.block_data(60_000 + i, B) for i in range(3)]
        cache.upsert_dirty_blocks({0: versions[0]})
        cache.submit_dirty_blocks([0], clone=True)   # the worker takes it and waits on the gate
        deadline = time.time() + 5
        while cache.flush_queue.qsize() and time.time() < deadline:
            time.sleep(0.01)
        cache.upsert_dirty_blocks({0: versions[1]})
        cache.submit_dirty_blocks([0], clone=True)   # queued
        cache.upsert_dirty_blocks({0: versions[2]})
        threading.Timer(0.3, st.gate.set).start()
        cache.submit_dirty_blocks([0], clone=True)   # queue full: synchronous, after the others
        cache.drain()
        assert torch.equal(st.read_blocks([0])[0], versions[2])
        assert cache.get_stats()["flush_queue_drops"] >= 1
        _assert_entries_consistent(cache)
    finally:
        st.gate.set()
        cache.shutdown()


class _SlowLog(BlockLogStore):
    def write_patch(self, block_dict):
        time.sleep(0.02)
        return super().write_patch(block_dict)


def test_full_slab_waits_for_flushes_instead_of_failing(tmp_path):
    """Every entry dirty or flushing behind a slow block log: new blocks wait
    for the flushes to return entries, and every block reads back current."""
    B, NB = 8, 24
    st = _SlowLog(str(tmp_path), B, NB, point_dim=G.POINT_DIM, verbose=False)
    cache = _cache(st, max_ram_gb=4 * B * G.POINT_DIM * 4 / 1024 ** 3, block_size=B,
                   capacity=8)
    want = {}
    try:
        for i in range(40):
            b = i % NB
            want[b] = G.block_data(70_000 + i, B)
            cache.upsert_dirty_blocks({b: want[b]})
        cache.drain()
        cache.flush_all_dirty()
        fresh = st.read_blocks(sorted(want))
        for b, t in want.items():
            assert torch.equal(fresh[b], t), b
        _assert_entries_consistent(cache)
    finally:
        cache.shutdown()
