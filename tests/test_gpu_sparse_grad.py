"""GPU: touched-only gradient accumulation (tidegs_b200/sparse_grad.py)
against the oracle restatement (oracle/sparse_grad.py, pinned to the
reference's torch operations of engine.py:1801-1826, 2434-2471)."""
import numpy as np
import pytest
import torch

from oracle import sparse_grad as sg
from tidegs_b200 import SparseGradAccumulator, _lib

pytestmark = pytest.mark.gpu


def _camera_grads(rng, n):
    return {k: (rng.standard_normal((n, w)) * 1e-3).astype(np.float32)
            for k, w in (("xyz", 3), ("opacity", 1), ("scaling", 3), ("rotation", 4),
                         ("shs", 48))}


@pytest.mark.parametrize("M,cams,max_n,lookup", [(5000, 7, 900, "map"), (5000, 7, 900, "search"),
                                                 (300_000, 16, 60_000, "map"), (40, 3, 40, "map")])
def test_accumulation_is_bit_exact(M, cams, max_n, lookup):
    rng = np.random.default_rng(M + cams)
    filters = [rng.choice(M, size=int(rng.integers(0, max_n)), replace=False)
               for _ in range(cams)]
    filters[1] = np.zeros(0, np.int64)
    l2g = rng.permutation(10 * M)[:M].astype(np.int64)
    acc = SparseGradAccumulator([torch.from_numpy(f).cuda() for f in filters], M,
                                torch.from_numpy(l2g).cuda())
    if lookup == "search":
        acc._pos_map = None  # binary search of the touched rows instead of the map
    touched = sg.touched_rows(filters, M)
    assert np.array_equal(acc.sparse_grad_local_ids.cpu().numpy(), touched)
    assert np.array_equal(acc.sparse_visibility_indices.numpy(), l2g[touched])
    want = sg.zero_components(touched.size)
    for cam, f in enumerate(filters):
        g = _camera_grads(rng, len(f))
        shs = None if cam == 2 else g["shs"]
        sg.accumulate(want, touched, f, g["xyz"], g["opacity"], g["scaling"], g["rotation"], shs)
        t = {k: torch.from_numpy(v).cuda() for k, v in g.items()}
        acc.add(torch.from_numpy(f).cuda(), t["xyz"], t["opacity"], t["scaling"], t["rotation"],
                None if shs is None else t["shs"])
    acc.check()
    for name in sg.WIDTHS:
        np.testing.assert_array_equal(acc.sparse_grad_components[name].cpu().numpy(), want[name],
                                      err_msg=name)


def test_repeated_ids_accumulate_with_atomics():
    """unique_filter=False: ids may repeat inside one filter; every addition
    lands (order of repeats unspecified: compare with a tolerance)."""
    rng = np.random.default_rng(3)
    M = 2000
    f = rng.integers(0, M, 5000)
    acc = SparseGradAccumulator([torch.from_numpy(f).cuda()], M)
    touched = sg.touched_rows([f], M)
    g = _camera_grads(rng, f.size)
    want = sg.zero_components(touched.size)
    sg.accumulate(want, touched, f, g["xyz"], g["opacity"], g["scaling"], g["rotation"], g["shs"])
    t = {k: torch.from_numpy(v).cuda() for k, v in g.items()}
    acc.add(torch.from_numpy(f).cuda(), t["xyz"], t["opacity"], t["scaling"], t["rotation"],
            t["shs"], unique_filter=False)
    acc.check()
    for name in sg.WIDTHS:
        np.testing.assert_allclose(acc.sparse_grad_components[name].cpu().numpy(), want[name],
                                   rtol=1e-5, atol=1e-8, err_msg=name)


def test_filter_id_outside_touched_rows_is_reported():
    acc = SparseGradAccumulator([torch.tensor([1, 5, 9], device="cuda")], 16)
    z = lambda w: torch.zeros((2, w), device="cuda")
    acc.add(torch.tensor([5, 7], device="cuda"), z(3), z(1), z(3), z(4))
    with pytest.raises(RuntimeError, match="not among the touched rows"):
        acc.check()


def test_filter_id_out_of_range_is_reported():
    with pytest.raises(RuntimeError, match="out of range"):
        SparseGradAccumulator([torch.tensor([0, 16], device="cuda")], 16)


def test_bitmap_list_large_is_ordered_and_complete():
    """tgs_bitmap_list at working-set size (33.5 M bits, ~30 % set, ragged
    tail) equals numpy's nonzero."""
    rng = np.random.default_rng(8)
    num_bits = 2048 * 16384 - 77
    words = (num_bits + 31) // 32
    raw = rng.integers(0, 2 ** 32, words, dtype=np.uint64).astype(np.uint32)
    raw &= rng.integers(0, 2 ** 32, words, dtype=np.uint64).astype(np.uint32)  # ~25 % of bits
    bits = np.unpackbits(raw.view(np.uint8), bitorder="little")[:num_bits]
    want = np.nonzero(bits)[0]
    bitmap = torch.from_numpy(raw.view(np.int32)).cuda()
    out = torch.empty(want.size + 1, dtype=torch.int64, device="cuda")
    lib = _lib.load()
    scratch = torch.empty(int(lib.tgs_bitmap_list_scratch_words(num_bits)), dtype=torch.int64,
                          device="cuda")
    pos_map = torch.full((num_bits,), -1, dtype=torch.int32, device="cuda")
    _lib.call("tgs_bitmap_list", bitmap.data_ptr(), num_bits, out[1:].data_ptr(),
              out[:1].data_ptr(), scratch.data_ptr(), pos_map.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    host = out.cpu().numpy()
    assert host[0] == want.size
    assert np.array_equal(host[1:], want)
    expect_map = np.full(num_bits, -1, np.int32)
    expect_map[want] = np.arange(want.size, dtype=np.int32)
    assert np.array_equal(pos_map.cpu().numpy(), expect_map)
