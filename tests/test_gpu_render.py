"""GPU: the render path (tidegs_b200.render) against the reference's gsplat
1.0.0 kernels compiled from its sources (oracle/_ref/gsplat, built by
oracle/build_ref.py; those comparisons skip when it is absent) and against
the float64 autograd oracle (oracle/render.py).

Tolerances: forward float32 outputs within rtol 1e-5 of the reference
kernels (same fp32 arithmetic up to FMA contraction and __expf), within
rtol 1e-4 of the float64 oracle; gradients within 1e-3 of the largest
gradient magnitude (atomic summation order, float32 recovery of the
transmittance); the culling decisions (radii) and last contributing ids may
differ on boundary cases only (>= 99.9 % equal); intersection keys, flatten
ids and offsets bit-exact given the same projection outputs."""
import numpy as np
import pytest
import torch

from oracle import render as orc

pytestmark = pytest.mark.gpu

W, H, TILE = 128, 96, 16


def _ref():
    from oracle import build_ref

    return build_ref.load_prebuilt_gsplat()


def _scene(N, C, seed, w=W, h=H):
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(N, 3, generator=g, dtype=torch.float64) * torch.tensor([8.0, 6.0, 6.0]) \
        + torch.tensor([-4.0, -3.0, 3.0])
    quats = torch.randn(N, 4, generator=g, dtype=torch.float64)
    scales = torch.exp(torch.randn(N, 3, generator=g, dtype=torch.float64) * 0.4 - 2.0)
    opac = torch.rand(C, N, generator=g, dtype=torch.float64) * 0.8 + 0.1
    colors = torch.rand(C, N, 3, generator=g, dtype=torch.float64)
    views = torch.stack([orc.look_at((0.3 * c, -0.2 * c, -1.0), (0.0, 0.0, 6.0), up=(0.0, -1.0, 0.0))
                         for c in range(C)])
    Ks = torch.stack([orc.intrinsics(w, h, 60.0 + 5 * c) for c in range(C)])
    return means, quats, scales, opac, colors, views, Ks


def _cuda32(*ts):
    return [t.to("cuda", torch.float32).contiguous() for t in ts]


def _close(a, b, rtol, what, atol=None):
    a = a.double().cpu()
    b = b.double().cpu()
    scale = float(b.abs().max()) if b.numel() else 0.0
    atol = rtol * max(scale, 1e-12) if atol is None else atol
    err = float((a - b).abs().max()) if a.numel() else 0.0
    assert err <= atol + 0.0, f"{what}: max error {err:.3e} > {atol:.3e} (scale {scale:.3e})"


def _project(means, quats, scales, views, Ks, **kw):
    from tidegs_b200.render import fully_fused_projection

    return fully_fused_projection(means, None, quats, scales, views, Ks, W, H, **kw)


def test_projection_against_reference_and_oracle():
    means, quats, scales, _, _, views, Ks = _scene(3000, 2, seed=1)
    m, q, s, v, k = _cuda32(means, quats, scales, views, Ks)
    m.requires_grad_(True), q.requires_grad_(True), s.requires_grad_(True)
    radii, means2d, depths, conics, comps = _project(m, q, s, v, k, calc_compensations=True)
    ok = radii > 0
    assert 0.2 < float(ok.float().mean()) < 0.99
    # float64 oracle
    o_radii, o_m2, o_d, o_con, o_comp = orc.project(means, quats, scales, views, Ks, W, H)
    agree = (radii.cpu().long() == o_radii)
    assert float(agree.float().mean()) >= 0.999
    both = (ok.cpu() & (o_radii > 0))
    _close(means2d.detach().cpu()[both], o_m2[both], 1e-5, "means2d vs oracle")
    _close(depths.detach().cpu()[both], o_d[both], 1e-5, "depths vs oracle")
    _close(conics.detach().cpu()[both], o_con[both], 1e-4, "conics vs oracle")
    _close(comps.detach().cpu()[both], o_comp[both], 1e-4, "compensations vs oracle")
    # gradients through autograd, with upstream gradients on the kept entries
    g = torch.Generator().manual_seed(7)
    w2 = torch.randn(means2d.shape, generator=g, dtype=torch.float64) * both[..., None]
    wd = torch.randn(depths.shape, generator=g, dtype=torch.float64) * both
    wc = torch.randn(conics.shape, generator=g, dtype=torch.float64) * both[..., None]
    wk = torch.randn(comps.shape, generator=g, dtype=torch.float64) * both
    loss = ((means2d * w2.cuda().float()).sum() + (depths * wd.cuda().float()).sum()
            + (conics * wc.cuda().float()).sum() + (comps * wk.cuda().float()).sum())
    loss.backward()
    mm, qq, ss = (t.clone().requires_grad_(True) for t in (means, quats, scales))
    _, a2, ad, ac, ak = orc.project(mm, qq, ss, views, Ks, W, H)
    ((a2 * w2).sum() + (ad * wd).sum() + (ac * wc).sum() + (ak * wk).sum()).backward()
    _close(m.grad, mm.grad, 1e-3, "v_means vs oracle")
    _close(q.grad, qq.grad, 1e-3, "v_quats vs oracle")
    _close(s.grad, ss.grad, 1e-3, "v_scales vs oracle")
    ref = _ref()
    if ref is None:
        pytest.skip("reference gsplat kernels not built")
    r_radii, r_m2, r_d, r_con, r_comp = ref.fully_fused_projection_fwd(
        m.detach(), None, q.detach(), s.detach(), v, k, W, H, 0.3, 0.01, 1e10, 0.0, True)
    assert float((r_radii == radii).float().mean()) >= 0.999
    both = (r_radii > 0) & ok
    _close(means2d.detach()[both], r_m2[both], 1e-5, "means2d vs reference")
    _close(conics.detach()[both], r_con[both], 1e-4, "conics vs reference")
    r_vm, _, r_vq, r_vs, _ = ref.fully_fused_projection_bwd(
        m.detach(), None, q.detach(), s.detach(), v, k, W, H, 0.3, r_radii, r_con, r_comp,
        w2.cuda().float().contiguous(), wd.cuda().float().contiguous(),
        wc.cuda().float().contiguous(), wk.cuda().float().contiguous(), False)
    _close(m.grad, r_vm, 1e-3, "v_means vs reference")
    _close(q.grad, r_vq, 1e-3, "v_quats vs reference")
    _close(s.grad, r_vs, 1e-3, "v_scales vs reference")


def _intersections(radii, means2d, depths, C):
    from tidegs_b200.render import isect_offset_encode, isect_tiles

    tw, th = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    tiles, ids, flat = isect_tiles(means2d, radii, depths, TILE, tw, th)
    offsets = isect_offset_encode(ids, C, tw, th)
    return tiles, ids, flat, offsets, tw, th


def test_intersections_match_reference_exactly():
    means, quats, scales, _, _, views, Ks = _scene(4000, 3, seed=2)
    m, q, s, v, k = _cuda32(means, quats, scales, views, Ks)
    radii, means2d, depths, _, _ = _project(m, q, s, v, k)
    tiles, ids, flat, offsets, tw, th = _intersections(radii, means2d, depths, 3)
    assert ids.numel() > 1000
    assert torch.all(ids[1:] >= ids[:-1])
    # offsets point at the first key of each (camera, tile)
    tile_of = (ids >> 32)
    bits = int(np.floor(np.log2(tw * th))) + 1
    flat_tile = (tile_of >> bits) * (tw * th) + (tile_of & ((1 << bits) - 1))
    expect = torch.searchsorted(flat_tile, torch.arange(3 * tw * th, device="cuda"))
    assert torch.equal(offsets.view(-1).long(), expect)
    # empty: nothing projected
    z = torch.zeros_like(radii)
    t0, i0, f0, o0, _, _ = _intersections(z, means2d, depths, 3)
    assert i0.numel() == 0 and f0.numel() == 0 and int(o0.abs().sum()) == 0 and int(t0.sum()) == 0
    ref = _ref()
    if ref is None:
        pytest.skip("reference gsplat kernels not built")
    r_tiles, r_ids, r_flat = ref.isect_tiles(means2d, radii, depths, None, None, 3, TILE, tw, th,
                                             True, True)
    assert torch.equal(tiles, r_tiles)
    assert torch.equal(ids, r_ids)
    assert torch.equal(flat, r_flat)
    assert torch.equal(offsets, ref.isect_offset_encode(r_ids, 3, tw, th))


def test_intersection_order_with_depth_ties_and_negative_depths():
    """Equal depths keep Gaussian order inside a tile; negative depths (and
    -0.0) sign-extend into the reference key and sort as its all-ones
    (camera, tile) bits. Checked against the reference's rule restated here
    (a stable sort of the written keys by their low 32 + tile + camera bits)
    and against the reference kernels."""
    from tidegs_b200.render import isect_tiles

    C, N = 3, 6000
    tw, th = (W + TILE - 1) // TILE, (H + TILE - 1) // TILE
    g = torch.Generator().manual_seed(11)
    means2d = (torch.rand((C, N, 2), generator=g) * torch.tensor([W * 1.2, H * 1.2])
               - torch.tensor([W * 0.1, H * 0.1])).cuda()
    radii = torch.randint(0, 40, (C, N), generator=g, dtype=torch.int32)
    radii[torch.rand((C, N), generator=g) < 0.2] = 0
    levels = torch.tensor([0.5, 1.0, 1.0, 2.5, 7.0, -0.0, -1.5, 3.0e-38, float("inf")])
    depths = levels[torch.randint(0, levels.numel(), (C, N), generator=g)].cuda()
    radii = radii.cuda()
    tiles, ids, flat = isect_tiles(means2d, radii, depths, TILE, tw, th)
    u_tiles, u_ids, u_flat = isect_tiles(means2d, radii, depths, TILE, tw, th, sort=False)
    assert torch.equal(tiles, u_tiles) and ids.numel() == u_ids.numel() > 10000
    bits = 32 + (int(np.floor(np.log2(tw * th))) + 1) + (int(np.floor(np.log2(C))) + 1)
    order = torch.sort(u_ids & ((1 << bits) - 1), stable=True).indices
    assert torch.equal(ids, u_ids[order])
    assert torch.equal(flat, u_flat[order])
    assert bool((ids < 0).any()), "no negative-depth keys were made"
    ref = _ref()
    if ref is None:
        pytest.skip("reference gsplat kernels not built")
    r_tiles, r_ids, r_flat = ref.isect_tiles(means2d, radii, depths, None, None, C, TILE, tw, th,
                                             True, True)
    assert torch.equal(ids, r_ids) and torch.equal(flat, r_flat)
    r_tiles, r_ids, r_flat = ref.isect_tiles(means2d, radii, depths, None, None, C, TILE, tw, th,
                                             False, True)
    assert torch.equal(u_ids, r_ids) and torch.equal(u_flat, r_flat)


def _render_inputs(N, C, seed, w=W, h=H):
    means, quats, scales, opac, colors, views, Ks = _scene(N, C, seed, w, h)
    m, q, s, v, k = _cuda32(means, quats, scales, views, Ks)
    return means, quats, scales, opac, colors, views, Ks, m, q, s, v, k


def test_rasterize_against_reference():
    means, quats, scales, opac, colors, views, Ks, m, q, s, v, k = _render_inputs(3000, 2, 3)
    radii, means2d, depths, conics, _ = _project(m, q, s, v, k)
    _, _, flat, offsets, tw, th = _intersections(radii, means2d, depths, 2)
    from tidegs_b200.render import rasterize_to_pixels

    col, op = _cuda32(colors, opac)
    bg = torch.tensor([[0.1, 0.2, 0.3], [0.0, 0.5, 1.0]], device="cuda")
    mm = means2d.detach().clone().requires_grad_(True)
    cc = conics.detach().clone().requires_grad_(True)
    co = col.clone().requires_grad_(True)
    oo = op.clone().requires_grad_(True)
    rc, ra = rasterize_to_pixels(mm, cc, co, oo, W, H, TILE, offsets, flat, backgrounds=bg,
                                 absgrad=True)
    assert 0.05 < float(ra.detach().mean()) < 0.999
    g = torch.Generator(device="cuda").manual_seed(5)
    vc = torch.randn(rc.shape, generator=g, device="cuda")
    va = torch.randn(ra.shape, generator=g, device="cuda")
    ((rc * vc).sum() + (ra * va).sum()).backward()
    ref = _ref()
    if ref is None:
        pytest.skip("reference gsplat kernels not built")
    r_rc, r_ra, r_last = ref.rasterize_to_pixels_fwd(means2d.detach(), conics.detach(), col, op, bg,
                                                     W, H, TILE, offsets, flat)
    _close(rc.detach(), r_rc, 1e-5, "render colors vs reference", atol=2e-5)
    _close(ra.detach(), r_ra, 1e-5, "render alphas vs reference", atol=2e-5)
    r_abs, r_vm, r_vc, r_vcol, r_vo = ref.rasterize_to_pixels_bwd(
        means2d.detach(), conics.detach(), col, op, bg, W, H, TILE, offsets, flat, r_ra, r_last,
        vc, va, True)
    _close(mm.grad, r_vm, 1e-3, "v_means2d vs reference")
    _close(mm.absgrad, r_abs, 1e-3, "|v_means2d| vs reference")
    _close(cc.grad, r_vc, 1e-3, "v_conics vs reference")
    _close(co.grad, r_vcol, 1e-3, "v_colors vs reference")
    _close(oo.grad, r_vo, 1e-3, "v_opacities vs reference")


def test_render_chain_against_oracle():
    """Projection -> intersections -> rasterization, forward and all input
    gradients, against the float64 oracle on the same intersection lists."""
    from tidegs_b200.render import rasterize_to_pixels

    global W, H
    w0, h0 = W, H
    W, H = 48, 40
    try:
        means, quats, scales, opac, colors, views, Ks, m, q, s, v, k = _render_inputs(
            220, 1, 4, 48, 40)
        for t in (m, q, s):
            t.requires_grad_(True)
        col, op = _cuda32(colors, opac)
        col.requires_grad_(True), op.requires_grad_(True)
        radii, means2d, depths, conics, _ = _project(m, q, s, v, k)
        _, _, flat, offsets, tw, th = _intersections(radii, means2d, depths, 1)
        rc, ra = rasterize_to_pixels(means2d, conics, col, op, W, H, TILE, offsets, flat)
        g = torch.Generator().manual_seed(9)
        wc = torch.randn(rc.shape, generator=g, dtype=torch.float64)
        wa = torch.randn(ra.shape, generator=g, dtype=torch.float64)
        ((rc * wc.cuda().float()).sum() + (ra * wa.cuda().float()).sum()).backward()

        mm, qq, ss, oo, cc = (t.clone().requires_grad_(True) for t in (means, quats, scales, opac,
                                                                         colors))
        _, o_m2, _, o_con, _ = orc.project(mm, qq, ss, views, Ks, W, H)
        o_rc, o_ra = orc.rasterize(o_m2, o_con, cc, oo, W, H, TILE, offsets.cpu(), flat.cpu())
        ((o_rc * wc).sum() + (o_ra * wa).sum()).backward()
        _close(rc.detach(), o_rc.detach(), 1e-4, "render colors vs oracle", atol=1e-4)
        _close(ra.detach(), o_ra.detach(), 1e-4, "render alphas vs oracle", atol=1e-4)
        _close(col.grad, cc.grad, 2e-3, "v_colors vs oracle")
        _close(op.grad, oo.grad, 2e-3, "v_opacities vs oracle")
        _close(m.grad, mm.grad, 2e-3, "v_means vs oracle")
        _close(q.grad, qq.grad, 2e-3, "v_quats vs oracle")
        _close(s.grad, ss.grad, 2e-3, "v_scales vs oracle")
    finally:
        W, H = w0, h0


@pytest.mark.parametrize("degree,K", [(0, 1), (1, 4), (2, 16), (3, 16), (4, 25)])
def test_spherical_harmonics_against_reference_and_oracle(degree, K):
    from tidegs_b200.render import spherical_harmonics

    g = torch.Generator().manual_seed(40 + degree)
    N = 3000
    dirs64 = torch.randn(2, N, 3, generator=g, dtype=torch.float64) * 5.0
    coeffs64 = torch.randn(2, N, K, 3, generator=g, dtype=torch.float64) * 0.3
    v64 = torch.randn(2, N, 3, generator=g, dtype=torch.float64)
    dirs, coeffs, v = _cuda32(dirs64, coeffs64, v64)
    d = dirs.clone().requires_grad_(True)
    c = coeffs.clone().requires_grad_(True)
    colors = spherical_harmonics(degree, d, c)
    colors.backward(v)
    # float64 oracle with autograd
    d64 = dirs.double().cpu().requires_grad_(True)
    c64 = coeffs.double().cpu().requires_grad_(True)
    ocol = orc.sh_colors(degree, d64, c64)
    ocol.backward(v.double().cpu())
    _close(colors.detach(), ocol.detach(), 1e-5, "SH colors vs oracle")
    _close(c.grad, c64.grad, 1e-5, "v_coeffs vs oracle")
    # degree 0 is constant in the direction: no gradient reaches dirs
    d64_grad = d64.grad if d64.grad is not None else torch.zeros_like(d64)
    _close(d.grad, d64_grad, 1e-4, "v_dirs vs oracle", atol=0.0 if degree == 0 else None)
    if K > (degree + 1) ** 2:
        assert torch.all(c.grad[..., (degree + 1) ** 2:, :] == 0)
    ref = _ref()
    if ref is None or not hasattr(ref, "compute_sh_fwd"):
        pytest.skip("reference gsplat SH kernels not built")
    r_col = ref.compute_sh_fwd(degree, dirs, coeffs, None)
    _close(colors.detach(), r_col, 1e-5, "SH colors vs reference")
    r_vc, r_vd = ref.compute_sh_bwd(K, degree, dirs, coeffs, None, v, True)
    _close(c.grad, r_vc, 1e-5, "v_coeffs vs reference")
    _close(d.grad, r_vd, 1e-4, "v_dirs vs reference")


def test_spherical_harmonics_masks_and_no_dir_gradient():
    from tidegs_b200.render import spherical_harmonics

    g = torch.Generator().manual_seed(5)
    dirs, coeffs, v = _cuda32(torch.randn(1000, 3, generator=g), torch.randn(1000, 16, 3, generator=g),
                              torch.randn(1000, 3, generator=g))
    masks = (torch.rand(1000, generator=g) < 0.6).cuda()
    c = coeffs.clone().requires_grad_(True)
    colors = spherical_harmonics(3, dirs, c, masks)  # dirs without grad: no v_dirs
    colors.backward(v)
    assert torch.all(colors[~masks] == 0) and torch.all(c.grad[~masks] == 0)
    full = spherical_harmonics(3, dirs, coeffs)
    assert torch.equal(colors[masks], full[masks])
    ref = _ref()
    if ref is None or not hasattr(ref, "compute_sh_bwd"):
        pytest.skip("reference gsplat SH kernels not built")
    r_vc, _ = ref.compute_sh_bwd(16, 3, dirs, coeffs, masks, v, False)
    _close(c.grad, r_vc, 1e-5, "masked v_coeffs vs reference")

