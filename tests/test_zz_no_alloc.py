"""GPU: the allocation-free compaction entry point.

tgs_global_to_local_compact_noalloc is for callers that cannot give the
library scratch memory when they call it (device memory planned once at
start-up, or a pipeline that cannot afford the device-wide synchronization
of cudaMalloc/cudaFree). It keeps its scratch in a fixed array inside the
library. This file is collected last (test_zz_*) so that a run stopping at
the first failure has already run every other test; it also passes on its
own in a fresh process, where its first call does the per-device set-up.

Its output is integer ids, so it must equal the allocating entry point's
output exactly, on two calls in a row (the second smaller than the first, so
stale scratch from the first call would show)."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_IDS = 1 << 25


def _inputs(n, seed, nb=4096, block_size=512):
    rng = np.random.default_rng(seed)
    starts = np.full(nb, -1, np.int64)
    present = rng.choice(nb, nb // 3, replace=False)
    starts[present] = rng.permutation(nb // 3) * block_size
    gids = rng.integers(-50, nb * block_size + 50, n).astype(np.int64)
    gids[::2] = present[rng.integers(0, present.size, gids[::2].size)] * block_size + \
        rng.integers(0, block_size, gids[::2].size)
    return (torch.from_numpy(gids).cuda(), torch.from_numpy(starts).cuda(), block_size)


def _with_caller_scratch(lib, gids, starts, block_size, stream):
    n = gids.numel()
    words = int(lib.tgs_compact_scratch_words(n))
    scratch = torch.empty(words, dtype=torch.int64, device="cuda")
    out = torch.full((n,), -99, dtype=torch.int64, device="cuda")
    count = torch.empty(1, dtype=torch.int64, device="cuda")
    assert lib.tgs_global_to_local_compact(out.data_ptr(), count.data_ptr(), gids.data_ptr(), n,
                                           starts.data_ptr(), starts.numel(), block_size,
                                           scratch.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    return out[: int(count.item())].cpu()


def _no_alloc(lib, gids, starts, block_size, stream):
    n = gids.numel()
    out = torch.full((n,), -99, dtype=torch.int64, device="cuda")
    count = torch.empty(1, dtype=torch.int64, device="cuda")
    rc = lib.tgs_global_to_local_compact_noalloc(out.data_ptr(), count.data_ptr(),
                                                 gids.data_ptr(), n, starts.data_ptr(),
                                                 starts.numel(), block_size, stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return out[: int(count.item())].cpu()


def test_no_alloc_matches_allocating_entry_point_on_two_calls():
    from tidegs_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for n, seed in ((3_000_001, 1), (70_001, 2)):
        gids, starts, bs = _inputs(n, seed)
        expect = _with_caller_scratch(lib, gids, starts, bs, stream)
        got = _no_alloc(lib, gids, starts, bs, stream)
        assert expect.numel() > 0
        assert torch.equal(got, expect)


def test_no_alloc_edge_sizes_match_allocating_entry_point():
    """No ids (count 0, nothing written) and exactly the largest accepted
    size, 33,554,432 ids, whose tile counts fill the whole fixed array."""
    from tidegs_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    count = torch.full((1,), 7, dtype=torch.int64, device="cuda")
    out = torch.full((4,), -99, dtype=torch.int64, device="cuda")
    starts = torch.full((8,), -1, dtype=torch.int64, device="cuda")
    assert lib.tgs_global_to_local_compact_noalloc(out.data_ptr(), count.data_ptr(), None, 0,
                                                   starts.data_ptr(), 8, 512, stream) == 0
    torch.cuda.synchronize()
    assert int(count.item()) == 0 and torch.all(out == -99)
    gids, starts, bs = _inputs(MAX_IDS, 3)
    expect = _with_caller_scratch(lib, gids, starts, bs, stream)
    got = _no_alloc(lib, gids, starts, bs, stream)
    assert expect.numel() > MAX_IDS // 3
    assert torch.equal(got, expect)
    del gids, starts


def test_no_alloc_rejects_sizes_beyond_its_fixed_scratch():
    from tidegs_b200 import _lib

    lib = _lib.load()
    count = torch.empty(1, dtype=torch.int64, device="cuda")
    dummy = torch.empty(1, dtype=torch.int64, device="cuda")
    rc = lib.tgs_global_to_local_compact_noalloc(dummy.data_ptr(), count.data_ptr(),
                                                 dummy.data_ptr(), MAX_IDS + 1,
                                                 dummy.data_ptr(), 1, 512, None)
    assert rc == 1
    assert "exceeds the fixed scratch limit" in _lib.last_error()
