"""CPU: argument handling of the render path's Python interface
(tidegs_b200.render, gsplat 1.0.0's signatures): shape errors raise
ValueError / NotImplementedError before any device work, and valid calls on
CPU tensors fail loudly (the path has no CPU fallback)."""
import pytest
import torch

from tidegs_b200 import render as tr


def test_spherical_harmonics_validates_shapes():
    dirs = torch.zeros(4, 3)
    with pytest.raises(ValueError, match="last dimension 3"):
        tr.spherical_harmonics(1, torch.zeros(4, 2), torch.zeros(4, 4, 3))
    with pytest.raises(ValueError, match="leading dimensions"):
        tr.spherical_harmonics(1, dirs, torch.zeros(5, 4, 3))
    with pytest.raises(ValueError, match="needs 16 coefficients"):
        tr.spherical_harmonics(3, dirs, torch.zeros(4, 9, 3))
    with pytest.raises(ValueError, match="degree 5"):
        tr.spherical_harmonics(5, dirs, torch.zeros(4, 36, 3))
    with pytest.raises(ValueError, match="masks"):
        tr.spherical_harmonics(1, dirs, torch.zeros(4, 4, 3), masks=torch.ones(3, dtype=torch.bool))


def test_render_calls_have_no_cpu_path():
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    with pytest.raises(RuntimeError, match="no CPU path"):
        tr.spherical_harmonics(1, torch.ones(4, 3), torch.zeros(4, 4, 3))
    with pytest.raises(RuntimeError, match="no CPU path"):
        tr.fully_fused_projection(torch.zeros(3, 3), None, torch.zeros(3, 4), torch.zeros(3, 3),
                                  torch.eye(4)[None], torch.eye(3)[None], 8, 8)


def test_unsupported_gsplat_options_raise():
    with pytest.raises(NotImplementedError, match="covars"):
        tr.fully_fused_projection(torch.zeros(3, 3), torch.zeros(3, 6), None, None,
                                  torch.eye(4)[None], torch.eye(3)[None], 8, 8)
    with pytest.raises(NotImplementedError, match="packed"):
        tr.fully_fused_projection(torch.zeros(3, 3), None, torch.zeros(3, 4), torch.zeros(3, 3),
                                  torch.eye(4)[None], torch.eye(3)[None], 8, 8, packed=True)
    with pytest.raises(NotImplementedError, match="packed"):
        tr.isect_tiles(torch.zeros(1, 3, 2), torch.zeros(1, 3, dtype=torch.int32),
                       torch.zeros(1, 3), 16, 1, 1, packed=True)
