"""Generates tests/golden/host_tier.json by running the reference's RAM block
cache (storage/tiered_cache_manager.py TieredCacheManager) and block log
(storage/log_storage_manager.py LogStorageManager) on seeded operation
sequences, recording the state after every operation.

    python tests/golden/make_host_tier_golden.py --reference <TideGS checkout>

Only this script imports the reference (by file path, nothing else of it is
executed); the tests replay the recorded operations on tidegs_b200's
PinnedBlockCache / BlockLogStore and compare the states.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
import tempfile
import threading
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
POINT_DIM = 59


def load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def block_data(seed: int, rows: int) -> torch.Tensor:
    """Deterministic block contents (the tests use the same function)."""
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((rows, POINT_DIM)).astype(np.float32))


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()[:16]


class RecordingStore:
    """Block store for the cache sequences: block b initially holds
    block_data(10_000 + b, B); write_patch stores the written tensors and
    logs (sorted ids, digests)."""

    def __init__(self, block_size: int):
        self.block_size = block_size
        self.data = {}
        self.writes = []
        self.lock = threading.Lock()

    def read_blocks(self, block_ids):
        with self.lock:
            return {int(b): self.data.get(int(b), block_data(10_000 + int(b), self.block_size)).clone()
                    for b in block_ids}

    def write_patch(self, blocks):
        with self.lock:
            ids = sorted(int(b) for b in blocks)
            self.writes.append([[b, digest(blocks[b])] for b in ids])
            for b in ids:
                self.data[b] = blocks[b].clone()
        return len(self.writes)


STAT_KEYS = ("cache_hits", "cache_misses", "evictions", "flushes", "prefetches",
             "async_flush_blocks", "sync_flush_blocks", "future_prefetch_blocks",
             "urgent_prefetch_blocks", "future_prefetch_submitted", "future_prefetch_skipped")


def cache_ops(seed: int, n_ops: int, n_blocks: int, block_size: int):
    rng = np.random.default_rng(seed)
    ops = []
    for i in range(n_ops):
        kind = rng.choice(["upsert_batch", "upsert", "prefetch", "prefetch", "submit",
                           "future", "evict", "flush_all"],
                          p=[0.2, 0.1, 0.3, 0.0, 0.12, 0.12, 0.08, 0.08])
        if kind in ("upsert_batch", "upsert"):
            ids = sorted(rng.choice(n_blocks, int(rng.integers(1, 5)), replace=False).tolist())
            rows = [int(rng.integers(1, block_size + 1)) if rng.random() < 0.2 else block_size
                    for _ in ids]
            ops.append({"op": kind, "blocks": ids, "rows": rows,
                        "seeds": [int(seed * 1000 + i * 10 + k) for k in range(len(ids))]})
        elif kind == "prefetch":
            ids = rng.choice(n_blocks, int(rng.integers(1, 7)), replace=True).tolist()
            ops.append({"op": kind, "blocks": [int(b) for b in ids]})
        elif kind == "submit":
            ids = sorted(rng.choice(n_blocks, int(rng.integers(1, 6)), replace=False).tolist())
            ops.append({"op": kind, "blocks": ids, "clone": bool(rng.random() < 0.5)})
        elif kind == "future":
            ids = sorted(rng.choice(n_blocks, int(rng.integers(1, 6)), replace=False).tolist())
            ops.append({"op": kind, "blocks": ids})
        elif kind == "evict":
            ops.append({"op": kind, "n": int(rng.integers(1, 4))})
        else:
            ops.append({"op": kind})
    return ops


def apply_cache_op(cache, op, block_size):
    """Runs one recorded operation; returns its result in JSON form."""
    kind = op["op"]
    if kind in ("upsert_batch", "upsert"):
        blocks = {b: block_data(s, r) for b, r, s in zip(op["blocks"], op["rows"], op["seeds"])}
        fn = cache.upsert_dirty_block_batch if kind == "upsert_batch" else cache.upsert_dirty_blocks
        return fn(blocks)
    if kind == "prefetch":
        got = cache.prefetch(op["blocks"])
        return {str(b): digest(t) for b, t in sorted(got.items())}
    if kind == "submit":
        return cache.submit_dirty_blocks(op["blocks"], clone=op["clone"])
    if kind == "future":
        return cache.prefetch_future(op["blocks"])
    if kind == "evict":
        cache.evict_and_flush(num_blocks=op["n"])
        return None
    cache.flush_all_dirty()
    return None


def cache_state(cache, store):
    cache.future_prefetch_queue.join()
    cache.flush_queue.join()
    with cache.cache_lock:
        order = [int(b) for b in cache.cache_data.keys()]
        content = {str(b): digest(t) for b, t in cache.cache_data.items()}
        dirty = sorted(int(b) for b in cache.dirty_set)
        versions = {str(b): int(v) for b, v in sorted(cache.block_versions.items())}
    with cache.flushing_lock:
        flushing = sorted(int(b) for b in cache.flushing_buffer)
    stats = cache.get_stats()
    return {"order": order, "content": content, "dirty": dirty, "versions": versions,
            "flushing": flushing, "stats": {k: int(stats[k]) for k in STAT_KEYS},
            "writes": len(store.writes)}


def run_cache_sequence(tcm, seed, n_ops=60, n_blocks=20, block_size=4, max_blocks=10):
    store = RecordingStore(block_size)
    max_ram_gb = max_blocks * block_size * POINT_DIM * 4 / (1024 ** 3)
    cache = tcm.TieredCacheManager(store, max_ram_gb=max_ram_gb, block_size=block_size,
                                   point_dim=POINT_DIM, verbose=False)
    ops = cache_ops(seed, n_ops, n_blocks, block_size)
    steps = []
    try:
        for op in ops:
            result = apply_cache_op(cache, op, block_size)
            steps.append({"result": result, **cache_state(cache, store)})
    finally:
        cache.shutdown()
    return {"seed": seed, "block_size": block_size, "max_ram_gb": max_ram_gb,
            "n_blocks": n_blocks, "ops": ops, "steps": steps, "writes": store.writes}


def run_log_sequence(lsm):
    B, NB = 4, 6
    out = {"block_size": B, "num_blocks": NB, "patches": []}
    with tempfile.TemporaryDirectory() as tmp:
        st = lsm.LogStorageManager(storage_dir=tmp, block_size=B, num_blocks=NB,
                                   point_dim=POINT_DIM, verbose=False, max_patch_files=64,
                                   max_patch_gb=0, min_free_gb=0)
        base = torch.cat([block_data(20_000 + b, B) for b in range(NB)])
        st.file_paths[0].write_bytes(base.numpy().tobytes())
        patches = [
            {1: (B, 1), 4: (B, 2)},
            {4: (B, 3), 0: (2, 4), 5: (B, 5)},
            {2: (0, 6), 1: (3, 7)},  # block 2: empty tensor, skipped
            {3: (B, 8)},
        ]
        for spec in patches:
            blocks = {b: (block_data(30_000 + s, r) if r else torch.empty((0, POINT_DIM)))
                      for b, (r, s) in spec.items()}
            pid = st.write_patch(blocks)
            path = st.file_paths[pid]
            index = {str(b): [loc.file_id, loc.offset, loc.size, loc.version]
                     for b, loc in sorted(st.index.items())}
            out["patches"].append({"spec": {str(b): list(v) for b, v in spec.items()},
                                   "patch_id": pid,
                                   "sha256": hashlib.sha256(path.read_bytes()).hexdigest(),
                                   "size": path.stat().st_size, "index": index})
        got = st.read_blocks([5, 0, 3, 1, 2, 4])
        out["read_order"] = [int(b) for b in got.keys()]
        out["read"] = {str(b): [list(t.shape), digest(t)] for b, t in got.items()}
        s = st.get_stats()
        out["stats"] = {k: int(s[k]) for k in ("reads", "writes", "patches_created", "num_patches",
                                               "live_patch_blocks", "total_files")}
        errors = {}
        for name, arg in (("bad_width", {0: torch.zeros((2, 3))}),
                          ("too_many_rows", {0: torch.zeros((B + 1, POINT_DIM))})):
            try:
                st.write_patch(arg)
                errors[name] = None
            except ValueError as exc:
                errors[name] = str(exc)
        try:
            st.read_blocks([NB + 3])
            errors["missing"] = None
        except ValueError as exc:
            errors["missing"] = str(exc)
        out["errors"] = errors
        st.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    root = Path(args.reference)
    tcm = load(root / "storage" / "tiered_cache_manager.py", "ref_tiered_cache_manager")
    lsm = load(root / "storage" / "log_storage_manager.py", "ref_log_storage_manager")
    fixture = {"log": run_log_sequence(lsm),
               "cache": [run_cache_sequence(tcm, seed) for seed in (1, 2, 3)]}
    (HERE / "host_tier.json").write_text(json.dumps(fixture, indent=None, separators=(",", ":")))
    print("wrote", HERE / "host_tier.json")


if __name__ == "__main__":
    main()
