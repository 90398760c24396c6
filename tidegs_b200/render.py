"""Render path before the optimizer, with gsplat 1.0.0's Python interface for
the five calls the engine makes (strategies/tide_engine/engine.py:481-561):
`fully_fused_projection`, `spherical_harmonics`, `isect_tiles`,
`isect_offset_encode` and `rasterize_to_pixels`, the projection, the SH
colors and the rasterization differentiable (autograd), so that
`from tidegs_b200.render import ...` replaces `from gsplat import ...`.

Kernels: tgs_project_fwd/bwd, tgs_sh_fwd/bwd, tgs_isect_count/write/offsets,
tgs_rasterize_fwd/bwd (libtidegs_b200.so). The sorted intersections come
from a stable sort of the Gaussians by depth and a stable sort of 32-bit
(camera, tile) keys (cub radix sorts, as gsplat sorts with cub) instead of
one sort of 64-bit keys; keys, flatten ids and their order are gsplat's.

Supported: gsplat's non-packed layout ([C, N, ...]), Gaussians given by
quats + scales, 1-4 color channels, no camera-pose gradients. Other options
raise (the engine uses none of them).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib

__all__ = ["fully_fused_projection", "isect_tiles", "isect_offset_encode", "rasterize_to_pixels",
           "rasterize_to_pixels_fwd", "rasterize_to_pixels_bwd", "spherical_harmonics"]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor; tidegs_b200 has no CPU path")
    return t.detach().to(torch.float32).contiguous()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _project_args(means, quats, scales, viewmats, Ks, width, height, eps2d, near, far, clip,
                  radii, means2d, depths, conics, comps) -> "_lib.ProjectArgs":
    a = _lib.ProjectArgs()
    a.means, a.quats, a.scales = means.data_ptr(), quats.data_ptr(), scales.data_ptr()
    a.viewmats, a.Ks = viewmats.data_ptr(), Ks.data_ptr()
    a.n_cameras, a.n_gaussians = int(viewmats.shape[0]), int(means.shape[0])
    a.image_width, a.image_height = int(width), int(height)
    a.eps2d, a.near_plane, a.far_plane, a.radius_clip = float(eps2d), float(near), float(far), float(clip)
    a.radii, a.means2d, a.depths, a.conics = (radii.data_ptr(), means2d.data_ptr(),
                                              depths.data_ptr(), conics.data_ptr())
    a.compensations = _ptr(comps)
    return a


class _Projection(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, viewmats, Ks, width, height, eps2d, near_plane,
                far_plane, radius_clip, calc_compensations):
        dev = means.device
        means_, quats_, scales_ = _f32(means, "means"), _f32(quats, "quats"), _f32(scales, "scales")
        view_, Ks_ = _f32(viewmats, "viewmats"), _f32(Ks, "Ks")
        C, N = int(view_.shape[0]), int(means_.shape[0])
        radii = torch.empty((C, N), dtype=torch.int32, device=dev)
        means2d = torch.empty((C, N, 2), dtype=torch.float32, device=dev)
        depths = torch.empty((C, N), dtype=torch.float32, device=dev)
        conics = torch.empty((C, N, 3), dtype=torch.float32, device=dev)
        comps = torch.empty((C, N), dtype=torch.float32, device=dev) if calc_compensations else None
        args = _project_args(means_, quats_, scales_, view_, Ks_, width, height, eps2d, near_plane,
                             far_plane, radius_clip, radii, means2d, depths, conics, comps)
        _lib.call("tgs_project_fwd", args, _stream(means_))
        ctx.save_for_backward(means_, quats_, scales_, view_, Ks_, radii, conics, comps)
        ctx.geom = (width, height, eps2d, near_plane, far_plane, radius_clip)
        ctx.mark_non_differentiable(radii)
        return radii, means2d, depths, conics, comps

    @staticmethod
    def backward(ctx, v_radii, v_means2d, v_depths, v_conics, v_comps):
        means, quats, scales, viewmats, Ks, radii, conics, comps = ctx.saved_tensors
        if ctx.needs_input_grad[3] or ctx.needs_input_grad[4]:
            raise NotImplementedError("gradients with respect to viewmats / Ks are not provided")
        width, height, eps2d, near, far, clip = ctx.geom
        C, N = radii.shape
        dev = means.device

        def grad_or_zeros(g, shape):
            return (torch.zeros(shape, dtype=torch.float32, device=dev) if g is None
                    else g.to(torch.float32).contiguous())

        v_means2d = grad_or_zeros(v_means2d, (C, N, 2))
        v_depths = grad_or_zeros(v_depths, (C, N))
        v_conics = grad_or_zeros(v_conics, (C, N, 3))
        v_comps = None if (v_comps is None or comps is None) else v_comps.to(torch.float32).contiguous()
        v_means = torch.zeros_like(means)
        v_quats = torch.zeros_like(quats)
        v_scales = torch.zeros_like(scales)
        b = _lib.ProjectBwdArgs()
        b.fwd = _project_args(means, quats, scales, viewmats, Ks, width, height, eps2d, near, far,
                              clip, radii, torch.empty(0, device=dev), torch.empty(0, device=dev),
                              conics, comps)
        b.v_means2d, b.v_depths, b.v_conics = (v_means2d.data_ptr(), v_depths.data_ptr(),
                                               v_conics.data_ptr())
        b.v_compensations = _ptr(v_comps)
        b.v_means, b.v_quats, b.v_scales = v_means.data_ptr(), v_quats.data_ptr(), v_scales.data_ptr()
        _lib.call("tgs_project_bwd", b, _stream(means))
        return (v_means, v_quats, v_scales, None, None, None, None, None, None, None, None, None)


def fully_fused_projection(means: torch.Tensor, covars: Optional[torch.Tensor],
                           quats: Optional[torch.Tensor], scales: Optional[torch.Tensor],
                           viewmats: torch.Tensor, Ks: torch.Tensor, width: int, height: int,
                           eps2d: float = 0.3, near_plane: float = 0.01, far_plane: float = 1e10,
                           radius_clip: float = 0.0, packed: bool = False,
                           sparse_grad: bool = False, calc_compensations: bool = False):
    """(radii [C,N] int32, means2d [C,N,2], depths [C,N], conics [C,N,3],
    compensations [C,N] or None) of every Gaussian in every camera; culled
    entries have radius 0 (gsplat 1.0.0 fully_fused_projection)."""
    if covars is not None or quats is None or scales is None:
        raise NotImplementedError("fully_fused_projection: Gaussians must be given by quats and "
                                  "scales (covars is not supported)")
    if packed or sparse_grad:
        raise NotImplementedError("fully_fused_projection: packed / sparse_grad are not supported")
    return _Projection.apply(means, quats, scales, viewmats, Ks, int(width), int(height), eps2d,
                             near_plane, far_plane, radius_clip, calc_compensations)


def isect_tiles(means2d: torch.Tensor, radii: torch.Tensor, depths: torch.Tensor, tile_size: int,
                tile_width: int, tile_height: int, sort: bool = True, packed: bool = False,
                n_cameras: Optional[int] = None, camera_ids=None, gaussian_ids=None
                ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(tiles_per_gauss [C,N] int32, isect_ids [n] int64, flatten_ids [n]
    int32): one key camera | tile | depth bits per overlapped tile, sorted
    (gsplat 1.0.0 isect_tiles)."""
    if packed:
        raise NotImplementedError("isect_tiles: packed is not supported")
    means2d_ = _f32(means2d, "means2d")
    depths_ = _f32(depths, "depths")
    radii_ = radii.detach().to(torch.int32).contiguous()
    C, N = int(means2d_.shape[0]), int(means2d_.shape[1])
    dev = means2d_.device
    n = C * N
    tiles = torch.empty((C, N), dtype=torch.int32, device=dev)
    s = _stream(means2d_)
    _lib.call("tgs_isect_count", means2d_.data_ptr(), radii_.data_ptr(), n, int(tile_size),
              int(tile_width), int(tile_height), tiles.data_ptr(), s)
    if not sort or n == 0:
        cum = torch.cumsum(tiles.view(-1), 0)
        n_isects = int(cum[-1].item()) if n else 0
        isect_ids = torch.empty(n_isects, dtype=torch.int64, device=dev)
        flatten_ids = torch.empty(n_isects, dtype=torch.int32, device=dev)
        if n_isects:
            _lib.call("tgs_isect_write", means2d_.data_ptr(), radii_.data_ptr(),
                      depths_.data_ptr(), n, N, int(tile_size), int(tile_width),
                      int(tile_height), cum.data_ptr(), isect_ids.data_ptr(),
                      flatten_ids.data_ptr(), s)
        return tiles, isect_ids, flatten_ids
    # sorted: Gaussians in depth order, their tiles emitted in that order with
    # 16- or 32-bit (camera, tile) keys, a stable sort of those, the 64-bit
    # keys put back
    order = torch.empty(n, dtype=torch.int32, device=dev)
    cum = torch.empty(n, dtype=torch.int64, device=dev)
    scratch = _scratch(dev, "tgs_isect_depth_order_scratch_bytes", n)
    _lib.call("tgs_isect_depth_order", depths_.data_ptr(), tiles.data_ptr(), n, order.data_ptr(),
              cum.data_ptr(), scratch.data_ptr(), scratch.numel(), s)
    del scratch
    n_isects = int(cum[-1].item())
    isect_ids = torch.empty(n_isects, dtype=torch.int64, device=dev)
    flatten_ids = torch.empty(n_isects, dtype=torch.int32, device=dev)
    if n_isects:
        key_bytes = int(_lib.load().tgs_isect_key_bytes(C, int(tile_width), int(tile_height)))
        if key_bytes == 0:
            raise RuntimeError("isect_tiles: camera and tile ids need more than 32 bits")
        key_dtype = torch.int16 if key_bytes == 2 else torch.int32
        keys = torch.empty(n_isects, dtype=key_dtype, device=dev)
        unsorted_ids = torch.empty(n_isects, dtype=torch.int32, device=dev)
        _lib.call("tgs_isect_write_ordered", means2d_.data_ptr(), radii_.data_ptr(),
                  depths_.data_ptr(), order.data_ptr(), n, N, int(tile_size), int(tile_width),
                  int(tile_height), cum.data_ptr(), keys.data_ptr(), unsorted_ids.data_ptr(), s)
        sorted_keys = torch.empty_like(keys)
        scratch = _scratch(dev, "tgs_isect_sort_tiles_scratch_bytes", n_isects, C,
                           int(tile_width), int(tile_height))
        _lib.call("tgs_isect_sort_tiles", keys.data_ptr(), unsorted_ids.data_ptr(), n_isects, C,
                  int(tile_width), int(tile_height), sorted_keys.data_ptr(),
                  flatten_ids.data_ptr(), scratch.data_ptr(), scratch.numel(), s)
        _lib.call("tgs_isect_expand_ids", sorted_keys.data_ptr(), key_bytes,
                  flatten_ids.data_ptr(), depths_.data_ptr(), n_isects, isect_ids.data_ptr(), s)
    return tiles, isect_ids, flatten_ids


def _scratch(dev: torch.device, query: str, *sizes) -> torch.Tensor:
    nbytes = ctypes.c_size_t(0)
    _lib.call(query, *sizes, ctypes.byref(nbytes))
    return torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)


def isect_offset_encode(isect_ids: torch.Tensor, n_cameras: int, tile_width: int,
                        tile_height: int) -> torch.Tensor:
    """[C, tile_height, tile_width] int32: index of the first sorted
    intersection of every (camera, tile) (gsplat 1.0.0 isect_offset_encode)."""
    dev = isect_ids.device
    offsets = torch.empty((int(n_cameras), int(tile_height), int(tile_width)), dtype=torch.int32,
                          device=dev)
    ids = isect_ids.detach().to(torch.int64).contiguous()
    _lib.call("tgs_isect_offsets", ids.data_ptr() if ids.numel() else None, int(ids.numel()),
              int(n_cameras), int(tile_width), int(tile_height), offsets.data_ptr(),
              torch.cuda.current_stream(dev).cuda_stream)
    return offsets


def _raster_args(means2d, conics, colors, opacities, backgrounds, width, height, tile_size,
                 offsets, flatten_ids, render_colors, render_alphas, last_ids) -> "_lib.RasterArgs":
    a = _lib.RasterArgs()
    a.means2d, a.conics, a.colors, a.opacities = (means2d.data_ptr(), conics.data_ptr(),
                                                  colors.data_ptr(), opacities.data_ptr())
    a.backgrounds = _ptr(backgrounds)
    a.n_cameras, a.n_gaussians, a.channels = (int(offsets.shape[0]), int(means2d.shape[1]),
                                              int(colors.shape[-1]))
    a.image_width, a.image_height, a.tile_size = int(width), int(height), int(tile_size)
    a.tile_height, a.tile_width = int(offsets.shape[1]), int(offsets.shape[2])
    a.tile_offsets = offsets.data_ptr()
    a.flatten_ids = _ptr(flatten_ids) if flatten_ids.numel() else None
    a.n_isects = int(flatten_ids.numel())
    a.render_colors, a.render_alphas, a.last_ids = (render_colors.data_ptr(),
                                                    render_alphas.data_ptr(), last_ids.data_ptr())
    return a


def rasterize_to_pixels_fwd(means2d, conics, colors, opacities, backgrounds, width: int,
                            height: int, tile_size: int, isect_offsets, flatten_ids):
    """(render_colors [C,H,W,D], render_alphas [C,H,W,1], last_ids [C,H,W]):
    the forward kernel alone, on contiguous float32 / int32 CUDA tensors
    (gsplat's rasterize_to_pixels_fwd binding)."""
    C, D = int(isect_offsets.shape[0]), int(colors.shape[-1])
    dev = means2d.device
    render_colors = torch.empty((C, height, width, D), dtype=torch.float32, device=dev)
    render_alphas = torch.empty((C, height, width, 1), dtype=torch.float32, device=dev)
    last_ids = torch.empty((C, height, width), dtype=torch.int32, device=dev)
    args = _raster_args(means2d, conics, colors, opacities, backgrounds, width, height, tile_size,
                        isect_offsets, flatten_ids, render_colors, render_alphas, last_ids)
    _lib.call("tgs_rasterize_fwd", args, _stream(means2d))
    return render_colors, render_alphas, last_ids


def rasterize_to_pixels_bwd(means2d, conics, colors, opacities, backgrounds, width: int,
                            height: int, tile_size: int, isect_offsets, flatten_ids, render_alphas,
                            last_ids, v_render_colors, v_render_alphas, absgrad: bool):
    """(v_means2d_abs or None, v_means2d, v_conics, v_colors, v_opacities):
    the backward kernel alone, on contiguous float32 / int32 CUDA tensors
    (gsplat's rasterize_to_pixels_bwd binding)."""
    dev = means2d.device
    v_means2d = torch.zeros_like(means2d)
    v_conics = torch.zeros_like(conics)
    v_colors = torch.zeros_like(colors)
    v_opac = torch.zeros_like(opacities)
    v_abs = torch.zeros_like(means2d) if absgrad else None
    b = _lib.RasterBwdArgs()
    b.fwd = _raster_args(means2d, conics, colors, opacities, backgrounds, width, height, tile_size,
                         isect_offsets, flatten_ids, torch.empty(0, device=dev), render_alphas,
                         last_ids)
    b.v_render_colors, b.v_render_alphas = v_render_colors.data_ptr(), v_render_alphas.data_ptr()
    b.v_means2d_abs = _ptr(v_abs)
    b.v_means2d, b.v_conics, b.v_colors, b.v_opacities = (v_means2d.data_ptr(), v_conics.data_ptr(),
                                                          v_colors.data_ptr(), v_opac.data_ptr())
    _lib.call("tgs_rasterize_bwd", b, _stream(means2d))
    return v_abs, v_means2d, v_conics, v_colors, v_opac


class _Rasterize(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2d, conics, colors, opacities, backgrounds, width, height, tile_size,
                isect_offsets, flatten_ids, absgrad):
        means2d_, conics_ = _f32(means2d, "means2d"), _f32(conics, "conics")
        colors_, opac_ = _f32(colors, "colors"), _f32(opacities, "opacities")
        bg_ = None if backgrounds is None else _f32(backgrounds, "backgrounds")
        offsets = isect_offsets.detach().to(torch.int32).contiguous()
        flat = flatten_ids.detach().to(torch.int32).contiguous()
        render_colors, render_alphas, last_ids = rasterize_to_pixels_fwd(
            means2d_, conics_, colors_, opac_, bg_, width, height, tile_size, offsets, flat)
        ctx.save_for_backward(means2d_, conics_, colors_, opac_, bg_, offsets, flat,
                              render_alphas, last_ids)
        ctx.shape = (width, height, tile_size, absgrad)
        ctx.means2d_input = means2d
        return render_colors, render_alphas

    @staticmethod
    def backward(ctx, v_render_colors, v_render_alphas):
        means2d, conics, colors, opac, bg, offsets, flat, render_alphas, last_ids = ctx.saved_tensors
        width, height, tile_size, absgrad = ctx.shape
        dev = means2d.device
        v_rc = (torch.zeros((offsets.shape[0], height, width, colors.shape[-1]), device=dev)
                if v_render_colors is None else v_render_colors.to(torch.float32).contiguous())
        v_ra = (torch.zeros_like(render_alphas) if v_render_alphas is None
                else v_render_alphas.to(torch.float32).contiguous())
        v_abs, v_means2d, v_conics, v_colors, v_opac = rasterize_to_pixels_bwd(
            means2d, conics, colors, opac, bg, width, height, tile_size, offsets, flat,
            render_alphas, last_ids, v_rc, v_ra, absgrad)
        if absgrad:
            ctx.means2d_input.absgrad = v_abs
        v_bg = None
        if ctx.needs_input_grad[4] and bg is not None:
            v_bg = (v_rc * (1.0 - render_alphas)).sum(dim=(1, 2))
        return (v_means2d, v_conics, v_colors, v_opac, v_bg, None, None, None, None, None, None)


def rasterize_to_pixels(means2d: torch.Tensor, conics: torch.Tensor, colors: torch.Tensor,
                        opacities: torch.Tensor, image_width: int, image_height: int,
                        tile_size: int, isect_offsets: torch.Tensor, flatten_ids: torch.Tensor,
                        backgrounds: Optional[torch.Tensor] = None, packed: bool = False,
                        absgrad: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """(render_colors [C,H,W,D], render_alphas [C,H,W,1]) by front-to-back
    alpha compositing of the tiles' sorted Gaussians (gsplat 1.0.0
    rasterize_to_pixels); differentiable in means2d, conics, colors,
    opacities and backgrounds."""
    if packed:
        raise NotImplementedError("rasterize_to_pixels: packed is not supported")
    D = int(colors.shape[-1])
    if not 1 <= D <= 4:
        raise ValueError(f"rasterize_to_pixels: 1 to 4 channels are supported (got {D})")
    C = int(isect_offsets.shape[0])
    th, tw = int(isect_offsets.shape[1]), int(isect_offsets.shape[2])
    if th * tile_size < image_height or tw * tile_size < image_width:
        raise ValueError("rasterize_to_pixels: the tile grid does not cover the image")
    N = int(means2d.shape[1])
    if means2d.shape != (C, N, 2) or conics.shape != (C, N, 3) or colors.shape[:2] != (C, N) \
            or opacities.shape != (C, N):
        raise ValueError("rasterize_to_pixels: inputs must be [C, N, ...] with C cameras")
    return _Rasterize.apply(means2d, conics, colors, opacities, backgrounds, int(image_width),
                            int(image_height), int(tile_size), isect_offsets, flatten_ids, absgrad)


class _SphericalHarmonics(torch.autograd.Function):
    @staticmethod
    def forward(ctx, degree, dirs, coeffs, masks):
        dirs_, coeffs_ = _f32(dirs, "dirs"), _f32(coeffs, "coeffs")
        masks_ = None if masks is None else masks.detach().to(torch.bool).contiguous()
        colors = torch.empty(dirs_.shape, dtype=torch.float32, device=dirs_.device)
        a = _sh_args(degree, dirs_, coeffs_, masks_)
        a.colors = colors.data_ptr()
        _lib.call("tgs_sh_fwd", a, _stream(dirs_))
        ctx.save_for_backward(dirs_, coeffs_, masks_)
        ctx.degree = degree
        return colors

    @staticmethod
    def backward(ctx, v_colors):
        dirs, coeffs, masks = ctx.saved_tensors
        v_colors = v_colors.to(torch.float32).contiguous()
        v_coeffs = torch.empty_like(coeffs)
        v_dirs = torch.empty_like(dirs) if ctx.needs_input_grad[1] else None
        b = _lib.ShBwdArgs()
        b.fwd = _sh_args(ctx.degree, dirs, coeffs, masks)
        b.v_colors, b.v_coeffs, b.v_dirs = v_colors.data_ptr(), v_coeffs.data_ptr(), _ptr(v_dirs)
        _lib.call("tgs_sh_bwd", b, _stream(dirs))
        return None, v_dirs, v_coeffs, None


def _sh_args(degree, dirs, coeffs, masks) -> "_lib.ShArgs":
    a = _lib.ShArgs()
    a.dirs, a.coeffs, a.masks = dirs.data_ptr(), coeffs.data_ptr(), _ptr(masks)
    a.n, a.K, a.degree = dirs.numel() // 3, int(coeffs.shape[-2]), int(degree)
    return a


def spherical_harmonics(degrees_to_use: int, dirs: torch.Tensor, coeffs: torch.Tensor,
                        masks: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[..., 3] colors from SH coefficients [..., K, 3] evaluated at the
    directions [..., 3] (normalized inside), using the first
    (degrees_to_use + 1)^2 coefficients; differentiable in dirs and coeffs
    (gsplat 1.0.0 spherical_harmonics). Masked-out entries (masks [...]
    False) give zero colors and zero gradients."""
    if dirs.shape[-1] != 3 or coeffs.shape[-1] != 3:
        raise ValueError("spherical_harmonics: dirs and coeffs must have last dimension 3")
    if coeffs.shape[:-2] != dirs.shape[:-1]:
        raise ValueError(f"spherical_harmonics: coeffs {tuple(coeffs.shape)} and dirs "
                         f"{tuple(dirs.shape)} do not share their leading dimensions")
    if not 0 <= degrees_to_use <= 4 or (degrees_to_use + 1) ** 2 > coeffs.shape[-2]:
        raise ValueError(f"spherical_harmonics: degree {degrees_to_use} needs "
                         f"{(degrees_to_use + 1) ** 2} coefficients, coeffs has "
                         f"{coeffs.shape[-2]}")
    if masks is not None and masks.shape != dirs.shape[:-1]:
        raise ValueError("spherical_harmonics: masks must have dirs' leading shape")
    return _SphericalHarmonics.apply(int(degrees_to_use), dirs, coeffs, masks)
