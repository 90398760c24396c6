"""GPU: the block-movement entry points at benchmark-scale block sizes,
against the numpy oracle (bit for bit) and through size-independent
properties (pack(unpack(x)) == x, copy idempotence)."""
import numpy as np
import pytest
import torch

from oracle import blocks as ob

pytestmark = pytest.mark.gpu

NAMES = ("xyz", "opacity", "scaling", "rotation", "features_dc", "features_rest")


def _empty(rows):
    return {n: torch.empty((rows, w), device="cuda") for n, w in ob.WIDTHS.items()}


@pytest.mark.parametrize("layout", ["cache", "unified"])
@pytest.mark.parametrize("rows,offset", [(16384 * 6 + 3, 0), (1000, 5), (3, 2), (64, 61)])
def test_unpack_pack_roundtrip(layout, rows, offset):
    from tidegs_b200 import _lib, _ops

    code = _lib.LAYOUT_CACHE if layout == "cache" else _lib.LAYOUT_UNIFIED
    gen = torch.Generator(device="cuda").manual_seed(rows)
    packed = torch.randn((rows, 59), generator=gen, device="cuda")
    comps = _empty(rows + offset)
    B = 4096
    nblk = (rows + B - 1) // B
    block_ids = torch.arange(100, 100 + nblk, device="cuda") * 3
    gids = torch.full((rows + offset,), -7, dtype=torch.int64, device="cuda")
    _ops.unpack_rows(packed, code, comps, offset, global_ids=gids, block_ids=block_ids,
                     block_size=B)
    host = packed.cpu().numpy()
    cols = ob.columns(layout)
    for n, w in ob.WIDTHS.items():
        np.testing.assert_array_equal(comps[n][offset:].cpu().numpy(), host[:, cols[n]:cols[n] + w])
    r = np.arange(rows)
    exp_g = block_ids.cpu().numpy()[r // B] * B + r % B
    np.testing.assert_array_equal(gids[offset:].cpu().numpy(), exp_g)
    assert (gids[:offset] == -7).all()
    out = torch.empty((rows, 59), device="cuda")
    _ops.pack_rows(comps, [offset], [rows], out, code)
    torch.cuda.synchronize()
    assert torch.equal(out, packed)


@pytest.mark.parametrize("layout", ["cache", "unified"])
@pytest.mark.parametrize("case", ["blocks", "ragged", "views"])
def test_pack_many_plans_against_oracle(layout, case):
    """Many plans: whole 16384-row blocks (bulk-staged tiles, more tiles than
    the persistent grid holds stages, so every stage is refilled), ragged
    counts and starts (plain-load tiles and short tail tiles), and component
    views whose bases are not 16-byte aligned (every tile on plain loads)."""
    from tidegs_b200 import _lib, _ops

    code = _lib.LAYOUT_CACHE if layout == "cache" else _lib.LAYOUT_UNIFIED
    rng = np.random.default_rng({"blocks": 1, "ragged": 2, "views": 3}[case])
    B = 16384
    if case == "blocks":
        nsrc = 160
        starts = (rng.permutation(nsrc)[:120] * B).tolist()
        counts = [B] * len(starts)
    else:
        nsrc = 40
        counts = rng.integers(1, 3 * 64 + 7, 300).tolist()
        starts = [int(rng.integers(0, nsrc * B - c)) for c in counts]
        counts[::7] = [64] * len(counts[::7])
        starts[::5] = [int(s) & ~3 for s in starts[::5]]
    rows = nsrc * B
    gen = torch.Generator(device="cuda").manual_seed(11)
    if case == "views":
        base = {n: torch.randn((rows + 1, w), generator=gen, device="cuda") for n, w in ob.WIDTHS.items()}
        comps = {n: base[n][1:] for n in NAMES}
        assert any(comps[n].data_ptr() % 16 for n in NAMES)
    else:
        comps = {n: torch.randn((rows, w), generator=gen, device="cuda") for n, w in ob.WIDTHS.items()}
    total = int(sum(counts))
    out_base = torch.full((total + 1, 59), -1.0, device="cuda")
    out = out_base[1:] if case == "ragged" else out_base[:total]
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    _ops.pack_rows(comps, starts, counts, out, code, err=err)
    torch.cuda.synchronize()
    assert err.tolist() == [0, 0, 0, 0]
    want = ob.pack_rows({n: comps[n].cpu().numpy() for n in NAMES}, starts, counts, layout)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    if case != "ragged":
        assert (out_base[total:] == -1).all()
    else:
        assert (out_base[0] == -1).all()


def test_unpack_misaligned_source_view():
    from tidegs_b200 import _lib, _ops

    base = torch.randn((1001, 59), device="cuda")
    packed = base.view(-1)[59 * 1 + 0:].view(1000, 59)  # 236-byte offset: not 16-aligned
    assert packed.data_ptr() % 16 != 0
    comps = _empty(1000)
    _ops.unpack_rows(packed, _lib.LAYOUT_CACHE, comps, 0)
    host = packed.cpu().numpy()
    for n, w in ob.WIDTHS.items():
        np.testing.assert_array_equal(comps[n].cpu().numpy(),
                                      host[:, ob.CACHE[n]:ob.CACHE[n] + w])


@pytest.mark.parametrize("aligned", [True, False])
def test_copy_blocks_against_oracle(aligned):
    from tidegs_b200 import _ops

    B = 16384
    nsrc = 24
    rng = np.random.default_rng(4)
    src = {n: torch.randn((nsrc * B, w), device="cuda") for n, w in ob.WIDTHS.items()}
    src_g = torch.arange(nsrc * B, device="cuda") * 7
    dst = {n: torch.zeros((nsrc * B + 64, w), device="cuda") for n, w in ob.WIDTHS.items()}
    dst_g = torch.zeros(nsrc * B + 64, dtype=torch.int64, device="cuda")
    picks = rng.permutation(nsrc)[:10]
    shift = 0 if aligned else 3
    src_starts = (picks * B + (0 if aligned else 1)).tolist()
    counts = [B - (0 if aligned else 5)] * 9 + [777]
    dst_starts = [k * B + shift for k in range(10)]
    _ops.copy_blocks(src, src_g, dst, dst_g, src_starts, dst_starts, counts, torch.device("cuda"))
    hs = {n: t.cpu().numpy() for n, t in src.items()}
    hd = {n: np.zeros((nsrc * B + 64, w), np.float32) for n, w in ob.WIDTHS.items()}
    hdg = np.zeros(nsrc * B + 64, np.int64)
    ob.copy_blocks(hs, src_g.cpu().numpy(), hd, hdg, src_starts, dst_starts, counts)
    for n in NAMES:
        np.testing.assert_array_equal(dst[n].cpu().numpy(), hd[n], err_msg=n)
    np.testing.assert_array_equal(dst_g.cpu().numpy(), hdg)


def test_block_bounds_and_starts_against_oracle():
    from tidegs_b200 import _ops

    B = 16384
    rng = np.random.default_rng(5)
    xyz = torch.from_numpy(rng.uniform(-100, 100, (40 * B, 3)).astype(np.float32)).cuda()
    starts = (rng.permutation(40)[:17] * B).tolist()
    counts = [B] * 16 + [123]
    out = torch.empty((17, 6), device="cuda")
    _ops.block_bounds(xyz, starts, counts, out)
    np.testing.assert_array_equal(out.cpu().numpy(),
                                  ob.block_bounds(xyz.cpu().numpy(), starts, counts))
    items = [(int(b), int(s)) for b, s in zip(rng.integers(-3, 5000, 700), rng.integers(0, 10**9, 700))]
    bs = _ops.build_block_starts(items, 4096, torch.device("cuda"))
    # duplicate ids: the reference's index_copy_ keeps one of them; use unique ids for parity
    uniq = {}
    for b, s in items:
        uniq.setdefault(b, s)
    items_u = list(uniq.items())
    bs = _ops.build_block_starts(items_u, 4096, torch.device("cuda"))
    np.testing.assert_array_equal(bs.cpu().numpy(), ob.build_block_starts(items_u, 4096))


def test_global_to_local_compact_large():
    from tidegs_b200 import _ops

    rng = np.random.default_rng(6)
    nb, B = 61036, 16384
    starts = np.full(nb, -1, np.int64)
    present = rng.choice(nb, 2048, replace=False)
    starts[present] = np.arange(2048) * B
    gids = rng.integers(-10, nb * B + 10, 3_000_000).astype(np.int64)
    gids[::3] = present[rng.integers(0, 2048, gids[::3].size)] * B + rng.integers(0, B, gids[::3].size)
    st = torch.from_numpy(starts).cuda()
    out = _ops.global_to_local_compact(torch.from_numpy(gids).cuda(), st, B)
    exp = ob.global_to_local(gids, starts, B)
    np.testing.assert_array_equal(out.cpu().numpy(), exp[exp >= 0])


def test_dirty_select_large_preserves_order():
    from tidegs_b200 import _ops

    rng = np.random.default_rng(8)
    nb = 61036
    bits = rng.random(nb) < 0.5
    words = np.zeros((nb + 31) // 32, np.uint32)
    for b in np.nonzero(bits)[0]:
        words[b >> 5] |= np.uint32(1) << np.uint32(b & 31)
    bitmap = torch.from_numpy(words.view(np.int32)).cuda()
    ids = sorted(set(rng.integers(0, nb, 20000).tolist()))
    got = _ops.dirty_select(bitmap, ids)
    assert got == [b for b in ids if bits[b]]
    assert _ops.dirty_list(bitmap, nb) == np.nonzero(bits)[0].tolist()


def test_dirty_mark_and_select_ignore_ids_outside_the_bitmap():
    """tgs_dirty_mark / tgs_dirty_select bound every id by the bitmap's
    block count: ids below 0 or past it are neither written nor read."""
    from tidegs_b200 import _lib

    nb = 40
    guard = torch.zeros(4, dtype=torch.int32, device="cuda")  # words 0-1: bitmap, 2-3: guard
    bitmap = guard[:2]
    ids = torch.tensor([3, -1, 39, 40, 63, 64, 1 << 40], dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("tgs_dirty_mark", bitmap.data_ptr(), nb, ids.data_ptr(), ids.numel(), 1, stream)
    words = guard.cpu().numpy().view(np.uint32)
    assert words[0] == (1 << 3) and words[1] == (1 << (39 - 32))
    assert words[2] == 0 and words[3] == 0
    out = torch.zeros(ids.numel() + 1, dtype=torch.int64, device="cuda")
    _lib.call("tgs_dirty_select", bitmap.data_ptr(), nb, ids.data_ptr(), ids.numel(),
              out[1:].data_ptr(), out[:1].data_ptr(), stream)
    host = out.cpu().numpy()
    assert host[1:1 + int(host[0])].tolist() == [3, 39]
