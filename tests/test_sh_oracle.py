"""CPU: the spherical-harmonics oracle (oracle/render.py sh_basis) pinned by
the mathematics it restates: the 25 basis functions of degree <= 4 are
orthonormal on the unit sphere (checked by a quadrature exact for
polynomials of degree <= 8: Gauss-Legendre in cos(theta) x uniform phi) and
take the closed-form zonal values on the z axis."""
import math

import numpy as np
import torch

from oracle import render as orc


def _sphere_quadrature(n_theta=12, n_phi=24):
    u, w = np.polynomial.legendre.leggauss(n_theta)  # u = cos(theta)
    phi = (np.arange(n_phi) + 0.5) * 2 * math.pi / n_phi
    ct, ph = np.meshgrid(u, phi, indexing="ij")
    st = np.sqrt(1 - ct * ct)
    dirs = np.stack([st * np.cos(ph), st * np.sin(ph), ct], -1).reshape(-1, 3)
    weights = np.repeat(w, n_phi) * (2 * math.pi / n_phi)
    return torch.from_numpy(dirs), torch.from_numpy(weights)


def test_sh_basis_is_orthonormal():
    dirs, w = _sphere_quadrature()
    # scaled, non-unit directions: the basis normalizes them
    Y = orc.sh_basis(4, dirs * 3.7)
    gram = (Y * w[:, None]).T @ Y
    assert torch.allclose(gram, torch.eye(25, dtype=torch.float64), atol=1e-9)


def test_sh_basis_zonal_values_on_the_axis():
    Y = orc.sh_basis(4, torch.tensor([[0.0, 0.0, 2.0]], dtype=torch.float64))[0]
    # Y_l0(z = 1) = sqrt((2l + 1) / (4 pi)), every m != 0 vanishes
    for l in range(5):
        for m in range(-l, l + 1):
            k = l * l + l + m
            expect = math.sqrt((2 * l + 1) / (4 * math.pi)) if m == 0 else 0.0
            assert abs(float(Y[k]) - expect) < 1e-12, (l, m)


def test_sh_colors_uses_the_first_coefficients_and_masks():
    g = torch.Generator().manual_seed(0)
    dirs = torch.randn(7, 3, generator=g, dtype=torch.float64)
    coeffs = torch.randn(7, 25, 3, generator=g, dtype=torch.float64)
    c2 = orc.sh_colors(2, dirs, coeffs)
    c2b = orc.sh_colors(2, dirs, coeffs[:, :9])
    assert torch.equal(c2, c2b)
    masks = torch.tensor([True, False] * 3 + [True])
    cm = orc.sh_colors(3, dirs, coeffs, masks)
    assert torch.all(cm[~masks] == 0) and torch.equal(cm[masks], orc.sh_colors(3, dirs, coeffs)[masks])
