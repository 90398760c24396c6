"""CPU oracle of the block frustum culling -- TEST INFRASTRUCTURE ONLY
(only tests/, __graft_entry__.smoke() and bench.py's baseline legs use it).

Restates storage/gaussian_block.py FrustumCuller (6-plane path) with every
float32 operation written out in the order numpy evaluates the reference's
expressions (sums strictly left to right):
  spheres  :286-298  center = (min+max)/2, radius = (sqrt(d.d)/2) * 1.15
  planes   :145-228  Gribb & Hartmann rows of proj @ view, each plane scaled
                     by 1/|(A, B, C)|
  cull     :429-465  visible iff dot(plane, (c, 1)) >= -radius for all six
  subset   :359-406  the same test over given ids, in their order
  order    :513-531  argsort of the squared center distances
Pinned by tests/golden/culling.npz, produced by running the reference's own
FrustumCuller on seeded scenes (tests/golden/make_culling_golden.py).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def spheres(bounds: np.ndarray):
    """(centers [N,3], radii [N]) float32."""
    b = np.asarray(bounds, dtype=F32)
    lo, hi = b[:, :3], b[:, 3:]
    centers = (lo + hi) / F32(2.0)
    d = hi - lo
    s = (d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2]
    radii = (np.sqrt(s) / F32(2.0)) * F32(1.15)
    return centers.astype(F32), radii.astype(F32)


def planes(view: np.ndarray, proj: np.ndarray) -> np.ndarray:
    """(6, 4) float32: left, right, bottom, top, near, far."""
    vp = np.asarray(proj) @ np.asarray(view)
    out = np.zeros((6, 4), dtype=F32)
    rows = [(0, +1), (0, -1), (1, +1), (1, -1), (2, +1), (2, -1)]
    for i, (k, sign) in enumerate(rows):
        out[i] = vp[3, :] + vp[k, :] if sign > 0 else vp[3, :] - vp[k, :]
    for i in range(6):
        # numpy float32 scalar powers, as the reference writes them: the scalar
        # power is not always the correctly rounded square (a * a)
        a, b, c = out[i, 0], out[i, 1], out[i, 2]
        n = np.sqrt(a ** 2 + b ** 2 + c ** 2)
        out[i] = out[i] / n
    return out


def visible(centers: np.ndarray, radii: np.ndarray, pl: np.ndarray, ids=None) -> np.ndarray:
    """Visible ids (ascending for ids=None, else in the order of ids)."""
    ids = np.arange(centers.shape[0]) if ids is None else np.asarray(ids, dtype=np.int64)
    c = centers[ids]
    neg_r = -radii[ids]
    ok = np.ones(ids.size, bool)
    for j in range(6):
        p = pl[j]
        d = ((p[0] * c[:, 0] + p[1] * c[:, 1]) + p[2] * c[:, 2]) + p[3]
        ok &= d >= neg_r
    return ids[ok]
