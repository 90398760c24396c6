"""CPU oracle of the render path before the optimizer -- TEST INFRASTRUCTURE
ONLY (only tests/, __graft_entry__.smoke() and bench.py's baseline legs use
it).

A float64 torch restatement of gsplat 1.0.0's projection and rasterization
(3D Gaussian splatting, Kerbl et al. 2023), whose backward is torch
autograd, so the CUDA kernels' hand-derived gradients are checked against
exact derivatives of the same forward:
  project    gsplat/cuda/csrc/fully_fused_projection_fwd.cu:19-121 (utils.cuh
             quat_to_rotmat, quat_scale_to_covar_preci, persp_proj, add_blur)
  rasterize  rasterize_to_pixels_fwd.cu:15-158 (front-to-back compositing,
             alpha = min(0.999, o exp(-sigma)), skipped below 1/255, a pixel
             stops when its transmittance would reach 1e-4)
  sh_colors  compute_sh_fwd.cu, spherical_harmonics.cuh:11-90 (real SH of
             degree <= 4 at the normalized direction)
Pinning: gsplat's Python reference (gsplat/cuda/_torch_impl.py) is not part
of the reference checkout, and its CUDA kernels run only on a GPU; the GPU
tests compare this oracle, tidegs_b200 and the reference kernels (compiled
from the reference sources by oracle/build_ref.py) with each other.
"""
from __future__ import annotations

import math

import torch

F64 = torch.float64


def quat_to_rotmat(quats: torch.Tensor) -> torch.Tensor:
    q = quats / quats.norm(dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    ], dim=-1).reshape(*q.shape[:-1], 3, 3)


def project(means, quats, scales, viewmats, Ks, width: int, height: int, eps2d=0.3,
            near_plane=0.01, far_plane=1e10, radius_clip=0.0):
    """(radii [C,N] int64, means2d [C,N,2], depths [C,N], conics [C,N,3],
    compensations [C,N]); entries with radius 0 are culled (their other
    outputs are still computed, for gradient checks)."""
    R = viewmats[:, :3, :3]
    t = viewmats[:, :3, 3]
    pc = torch.einsum("cij,nj->cni", R, means) + t[:, None, :]
    Rq = quat_to_rotmat(quats)
    M = Rq * scales[:, None, :]
    cov = M @ M.transpose(-1, -2)
    cov_c = R[:, None] @ cov[None] @ R.transpose(-1, -2)[:, None]
    fx, fy = Ks[:, 0, 0][:, None], Ks[:, 1, 1][:, None]
    cx, cy = Ks[:, 0, 2][:, None], Ks[:, 1, 2][:, None]
    x, y, z = pc.unbind(-1)
    lim_x = 1.3 * (0.5 * width / fx)
    lim_y = 1.3 * (0.5 * height / fy)
    rz = 1.0 / z
    tx = z * torch.minimum(lim_x, torch.maximum(-lim_x, x * rz))
    ty = z * torch.minimum(lim_y, torch.maximum(-lim_y, y * rz))
    zero = torch.zeros_like(z)
    J = torch.stack([fx * rz, zero, -fx * tx * rz * rz,
                     zero, fy * rz, -fy * ty * rz * rz], dim=-1).reshape(*z.shape, 2, 3)
    cov2d = J @ cov_c @ J.transpose(-1, -2)
    det_orig = cov2d[..., 0, 0] * cov2d[..., 1, 1] - cov2d[..., 0, 1] * cov2d[..., 1, 0]
    eye = torch.eye(2, dtype=cov2d.dtype)
    cov2d = cov2d + eps2d * eye
    det = cov2d[..., 0, 0] * cov2d[..., 1, 1] - cov2d[..., 0, 1] * cov2d[..., 1, 0]
    conics = torch.stack([cov2d[..., 1, 1] / det, -cov2d[..., 0, 1] / det, cov2d[..., 0, 0] / det],
                         dim=-1)
    comps = torch.sqrt(torch.clamp(det_orig / det, min=0.0))
    means2d = torch.stack([fx * x * rz + cx, fy * y * rz + cy], dim=-1)
    with torch.no_grad():
        b = 0.5 * (cov2d[..., 0, 0] + cov2d[..., 1, 1])
        v1 = b + torch.sqrt(torch.clamp(b * b - det, min=0.01))
        radius = torch.ceil(3.0 * torch.sqrt(v1))
        mx, my = means2d[..., 0], means2d[..., 1]
        ok = ((z >= near_plane) & (z <= far_plane) & (det > 0) & (radius > radius_clip)
              & (mx + radius > 0) & (mx - radius < width) & (my + radius > 0)
              & (my - radius < height))
        radii = torch.where(ok, radius, torch.zeros_like(radius)).to(torch.int64)
    return radii, means2d, z, conics, comps


def rasterize(means2d, conics, colors, opacities, width: int, height: int, tile_size: int,
              isect_offsets, flatten_ids, backgrounds=None):
    """(render_colors [C,H,W,D], render_alphas [C,H,W,1]) from the sorted
    intersection lists (the same offsets / flatten ids the kernel uses),
    differentiable in means2d, conics, colors, opacities."""
    C, th, tw = isect_offsets.shape
    D = colors.shape[-1]
    n_isects = flatten_ids.numel()
    flat_m = means2d.reshape(-1, 2)
    flat_c = conics.reshape(-1, 3)
    flat_col = colors.reshape(-1, D)
    flat_o = opacities.reshape(-1)
    offs = isect_offsets.reshape(-1).tolist()
    fid = flatten_ids.tolist()
    out_rows = []
    alpha_rows = []
    for cam in range(C):
        img = [[None] * tw for _ in range(th)]
        alp = [[None] * tw for _ in range(th)]
        for ty in range(th):
            for tx in range(tw):
                k = cam * th * tw + ty * tw + tx
                start = offs[k]
                end = offs[k + 1] if k + 1 < len(offs) else n_isects
                ys = torch.arange(ty * tile_size, ty * tile_size + tile_size, dtype=F64)
                xs = torch.arange(tx * tile_size, tx * tile_size + tile_size, dtype=F64)
                py, px = torch.meshgrid(ys + 0.5, xs + 0.5, indexing="ij")
                px, py = px.reshape(-1), py.reshape(-1)
                T = torch.ones_like(px)
                acc = torch.zeros((px.numel(), D), dtype=F64)
                done = torch.zeros(px.numel(), dtype=torch.bool)
                for idx in range(start, end):
                    g = fid[idx]
                    dx = flat_m[g, 0] - px
                    dy = flat_m[g, 1] - py
                    c = flat_c[g]
                    sigma = 0.5 * (c[0] * dx * dx + c[2] * dy * dy) + c[1] * dx * dy
                    alpha = torch.clamp(flat_o[g] * torch.exp(-sigma), max=0.999)
                    use = (~done) & (sigma >= 0) & (alpha >= 1.0 / 255.0)
                    next_T = T * (1.0 - alpha)
                    stop = use & (next_T <= 1e-4)
                    use = use & ~stop
                    done = done | stop
                    acc = acc + torch.where(use[:, None], (alpha * T)[:, None] * flat_col[g][None],
                                            torch.zeros_like(acc))
                    T = torch.where(use, next_T, T)
                color = acc
                if backgrounds is not None:
                    color = color + T[:, None] * backgrounds[cam][None]
                img[ty][tx] = color.reshape(tile_size, tile_size, D)
                alp[ty][tx] = (1.0 - T).reshape(tile_size, tile_size, 1)
        full = torch.cat([torch.cat(row, dim=1) for row in img], dim=0)[:height, :width]
        fa = torch.cat([torch.cat(row, dim=1) for row in alp], dim=0)[:height, :width]
        out_rows.append(full)
        alpha_rows.append(fa)
    return torch.stack(out_rows), torch.stack(alpha_rows)


def sh_basis(degree: int, dirs: torch.Tensor) -> torch.Tensor:
    """[..., (degree + 1)^2] real SH basis at dirs / |dirs| (float64), in the
    order and signs 3D Gaussian splatting and gsplat use
    (spherical_harmonics.cuh:11-90); the forms follow the reference's own
    Sloan-style recurrences (products of z-polynomials with the cos / sin
    multiple-angle terms C_m, S_m of (x, y)), not the closed polynomials the
    CUDA kernel uses, so the two are independent restatements."""
    n = dirs / dirs.norm(dim=-1, keepdim=True)
    x, y, z = n.unbind(-1)
    out = [torch.full_like(x, 0.28209479177387814)]
    if degree >= 1:
        out += [-0.48860251190292 * y, 0.48860251190292 * z, -0.48860251190292 * x]
    if degree >= 2:
        z2 = z * z
        c1, s1 = x * x - y * y, 2 * x * y
        t0b = -1.092548430592079 * z
        sh6 = 0.9461746957575601 * z2 - 0.3153915652525201
        out += [0.5462742152960395 * s1, t0b * y, sh6, t0b * x, 0.5462742152960395 * c1]
    if degree >= 3:
        c2, s2 = x * c1 - y * s1, x * s1 + y * c1
        t0c = -2.285228997322329 * z2 + 0.4570457994644658
        t1b = 1.445305721320277 * z
        sh12 = z * (1.865881662950577 * z2 - 1.119528997770346)
        out += [-0.5900435899266435 * s2, t1b * s1, t0c * y, sh12, t0c * x, t1b * c1,
                -0.5900435899266435 * c2]
    if degree >= 4:
        c3, s3 = x * c2 - y * s2, x * s2 + y * c2
        t0d = z * (-4.683325804901025 * z2 + 2.007139630671868)
        t1c = 3.31161143515146 * z2 - 0.47308734787878
        t2b = -1.770130769779931 * z
        sh20 = 1.984313483298443 * z * sh12 - 1.006230589874905 * sh6
        out += [0.6258357354491763 * s3, t2b * s2, t1c * s1, t0d * y, sh20, t0d * x, t1c * c1,
                t2b * c2, 0.6258357354491763 * c3]
    return torch.stack(out, dim=-1)


def sh_colors(degree: int, dirs: torch.Tensor, coeffs: torch.Tensor, masks=None) -> torch.Tensor:
    """[..., 3] = sum_k coeffs[..., k, :] Y_k (compute_sh_fwd.cu), zero where
    masks is False; differentiable (autograd gives the reference backward)."""
    K = (degree + 1) ** 2
    col = (sh_basis(degree, dirs)[..., None] * coeffs[..., :K, :]).sum(dim=-2)
    if masks is not None:
        col = torch.where(masks[..., None], col, torch.zeros_like(col))
    return col


def look_at(eye, target, up=(0.0, 0.0, 1.0)) -> torch.Tensor:
    """4x4 world-to-camera matrix of a camera at `eye` looking at `target`
    (camera z forward, OpenCV convention as the renderer uses)."""
    eye = torch.as_tensor(eye, dtype=F64)
    f = torch.as_tensor(target, dtype=F64) - eye
    f = f / f.norm()
    r = torch.linalg.cross(f, torch.as_tensor(up, dtype=F64))
    r = r / r.norm()
    d = torch.linalg.cross(f, r)
    R = torch.stack([r, d, f])
    m = torch.eye(4, dtype=F64)
    m[:3, :3] = R
    m[:3, 3] = -R @ eye
    return m


def intrinsics(width: int, height: int, fov_deg: float) -> torch.Tensor:
    f = 0.5 * width / math.tan(math.radians(fov_deg) / 2)
    return torch.tensor([[f, 0.0, width / 2], [0.0, f, height / 2], [0.0, 0.0, 1.0]], dtype=F64)
