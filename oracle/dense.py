"""CPU restatements of the masked dense optimizers -- test infrastructure only.

selective_adam: submodules/clm_kernels/adam.cu:29-40 (optimizer.py:46-87 calls
  it once per group). Rows with visibility[r] set are updated; no bias
  correction. Evaluated in numpy float32 with the C expression's operation
  order, one rounding per operation.
sophia: Sophia, Algorithm 3 of Liu et al. 2023 ("Sophia: A Scalable Stochastic
  Second-order Optimizer for Language Model Pre-training"), restated with
  h_hat = (u*g)^2, masked per row. TideGS has no Sophia: parity unpinned.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _row_mask(visibility: np.ndarray, shape) -> np.ndarray:
    vis = np.asarray(visibility).reshape(-1).astype(bool)
    n = vis.size
    width = int(np.prod(shape)) // n
    return np.repeat(vis, width).reshape(shape)


def selective_adam(param, grad, m, v, visibility, lr, beta1, beta2, eps):
    """In-place on param/m/v (float32 arrays of equal shape)."""
    mask = _row_mask(visibility, param.shape)
    b1, b2, e, one = F32(beta1), F32(beta2), F32(eps), F32(1.0)
    g = grad[mask]
    mm = b1 * m[mask] + (one - b1) * g
    vv = b2 * v[mask] + ((one - b2) * g) * g
    step = ((-F32(lr)) * mm) / (np.sqrt(vv) + e)
    param[mask] = param[mask] + step
    m[mask] = mm
    v[mask] = vv


def sophia(param, grad, m, h, visibility, lr, beta1, beta2, rho, eps, weight_decay=0.0,
           hessian_step=False, noise=None):
    """In-place on param/m/h."""
    mask = _row_mask(visibility, param.shape)
    b1, b2, one = F32(beta1), F32(beta2), F32(1.0)
    g = grad[mask]
    mm = b1 * m[mask] + (one - b1) * g
    hh = h[mask]
    if hessian_step:
        q = noise[mask] * g
        hh = b2 * hh + (one - b2) * (q * q)
    p = param[mask]
    if weight_decay != 0.0:
        p = p - (F32(lr) * F32(weight_decay)) * p
    ratio = mm / np.maximum(F32(rho) * hh, F32(eps))
    ratio = np.minimum(np.maximum(ratio, F32(-1.0)), F32(1.0))
    param[mask] = p - F32(lr) * ratio
    m[mask] = mm
    h[mask] = hh
