"""GPU parity of SelectiveAdam (reference optimizer.py:5-87 +
clm_kernels/adam.cu) and SelectiveSophia against the numpy oracle, bit for
bit (both sides round each fp32 operation once)."""
import numpy as np
import pytest
import torch

from oracle import dense

pytestmark = pytest.mark.gpu


def _groups(N, widths, seed, lrs):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    groups = []
    for w, lr in zip(widths, lrs):
        p = torch.randn((N, w), generator=gen, device="cuda")
        p.grad = torch.randn((N, w), generator=gen, device="cuda") * 1e-3
        groups.append({"params": [p], "lr": lr})
    return groups


@pytest.mark.parametrize("N", [1, 7, 1000, 262_147])
def test_selective_adam_all_groups_one_launch(N):
    from tidegs_b200 import SelectiveAdam

    widths = (3, 3, 45, 1, 3, 4)
    lrs = (1.6e-4, 2.5e-3, 1.25e-4, 0.05, 5e-3, 1e-3)
    groups = _groups(N, widths, N, lrs)
    ref = [(g["params"][0].detach().cpu().numpy().copy(), g["params"][0].grad.cpu().numpy())
           for g in groups]
    opt = SelectiveAdam(groups, eps=1e-15, betas=(0.9, 0.999))
    gen = torch.Generator(device="cuda").manual_seed(1)
    ms = [np.zeros_like(p) for p, _ in ref]
    vs = [np.zeros_like(p) for p, _ in ref]
    for step in range(3):
        vis = torch.rand(N, generator=gen, device="cuda") < 0.3
        opt.step(vis)
        for (p, g), m, v, lr in zip(ref, ms, vs, lrs):
            dense.selective_adam(p, g, m, v, vis.cpu().numpy(), lr, 0.9, 0.999, 1e-15)
    for grp, (p, _), m, v in zip(groups, ref, ms, vs):
        param = grp["params"][0]
        np.testing.assert_array_equal(param.detach().cpu().numpy(), p)
        st = opt.state[param]
        np.testing.assert_array_equal(st["exp_avg"].cpu().numpy(), m)
        np.testing.assert_array_equal(st["exp_avg_sq"].cpu().numpy(), v)


def test_selective_adam_unaligned_views_and_float_mask():
    from tidegs_b200 import SelectiveAdam

    N = 1001
    base = torch.randn(N * 3 + 1, device="cuda")
    p = torch.nn.Parameter(base[1:].view(N, 3).clone())  # contiguous copy
    view = base[1:].view(N, 3)                           # 4-byte offset storage
    view.grad = torch.randn((N, 3), device="cuda")
    p.grad = view.grad.clone()
    ref_p = view.detach().cpu().numpy().copy()
    opt = SelectiveAdam([{"params": [view], "lr": 0.01}], eps=1e-8, betas=(0.9, 0.999))
    mask = (torch.arange(N, device="cuda") % 3 == 0).float()
    opt.step(mask)
    m = np.zeros_like(ref_p)
    v = np.zeros_like(ref_p)
    dense.selective_adam(ref_p, view.grad.cpu().numpy(), m, v, mask.cpu().numpy() != 0, 0.01,
                         0.9, 0.999, 1e-8)
    np.testing.assert_array_equal(view.detach().cpu().numpy(), ref_p)


@pytest.mark.parametrize("wd", [0.0, 0.1])
def test_sophia_matches_oracle_with_hessian_refresh(wd):
    from tidegs_b200 import SelectiveSophia

    N = 50_003
    widths = (3, 45, 1)
    lrs = (1e-3, 2e-4, 5e-2)
    groups = _groups(N, widths, 3, lrs)
    ref = [(g["params"][0].detach().cpu().numpy().copy(), g["params"][0].grad.cpu().numpy())
           for g in groups]
    opt = SelectiveSophia(groups, betas=(0.965, 0.99), rho=0.04, eps=1e-15, weight_decay=wd, k=3)
    ms = [np.zeros_like(p) for p, _ in ref]
    hs = [np.zeros_like(p) for p, _ in ref]
    gen = torch.Generator(device="cuda").manual_seed(2)
    for t in range(1, 8):
        vis = torch.rand(N, generator=gen, device="cuda") < 0.3
        noise = [torch.randn(g["params"][0].shape, generator=gen, device="cuda") for g in groups]
        opt.step(vis, noise=noise)
        hess = (t % 3) == 1
        for (p, g), m, h, u, lr in zip(ref, ms, hs, noise, lrs):
            dense.sophia(p, g, m, h, vis.cpu().numpy(), lr, 0.965, 0.99, 0.04, 1e-15, wd,
                         hessian_step=hess, noise=u.cpu().numpy())
    for grp, (p, _), m, h in zip(groups, ref, ms, hs):
        param = grp["params"][0]
        np.testing.assert_array_equal(param.detach().cpu().numpy(), p)
        np.testing.assert_array_equal(opt.state[param]["exp_avg"].cpu().numpy(), m)
        np.testing.assert_array_equal(opt.state[param]["hessian"].cpu().numpy(), h)


def _close_1e6(actual, expected, what):
    """|a-b| <= 1e-6*|b| + 1e-6*max|b|: 1e-6 relative per element, and 1e-6
    of the tensor's scale where a value lands near zero by cancellation
    (p - step with p ~ step), where per-element relative error is
    meaningless."""
    scale = float(expected.abs().max())
    torch.testing.assert_close(actual, expected, rtol=1e-6, atol=1e-6 * scale, msg=what)


def test_selective_adam_matches_reference_cuda_kernel():
    """Against the reference's own submodules/clm_kernels/adam.cu, compiled
    for sm_100a into oracle/_ref by oracle/build_ref.py. The reference is
    built with nvcc's default FMA contraction, ours rounds every operation,
    so results differ by a few ulps; tolerance as in _close_1e6."""
    from oracle import build_ref
    from tidegs_b200 import SelectiveAdam

    ref = build_ref.load_prebuilt()
    if ref is None:
        pytest.skip("reference kernel not built (oracle/_ref)")
    N = 200_003
    widths = (3, 45, 1, 4)
    lrs = (1.6e-4, 1.25e-4, 0.05, 1e-3)
    groups = _groups(N, widths, 11, lrs)
    mirror = []
    for g in groups:
        p = g["params"][0]
        mirror.append((p.detach().clone(), p.grad.clone(), torch.zeros_like(p), torch.zeros_like(p)))
    opt = SelectiveAdam(groups, eps=1e-15, betas=(0.9, 0.999))
    gen = torch.Generator(device="cuda").manual_seed(5)
    for step in range(4):
        vis = torch.rand(N, generator=gen, device="cuda") < 0.3
        opt.step(vis)
        for (p, g, m, v), lr, w in zip(mirror, lrs, widths):
            ref.selective_adam_update(p, g, m, v, vis, lr, 0.9, 0.999, 1e-15, N, w)
    torch.cuda.synchronize()
    for grp, (p, _, m, v) in zip(groups, mirror):
        param = grp["params"][0]
        _close_1e6(param.detach(), p, "param")
        _close_1e6(opt.state[param]["exp_avg"], m, "exp_avg")
        _close_1e6(opt.state[param]["exp_avg_sq"], v, "exp_avg_sq")
