"""Masked (selective) optimizers and the resident-Adam metadata context
(drop-in for TideGS's optimizer.py).

* SelectiveAdam (optimizer.py:5-87): same constructor and step(visibility).
  The reference launches clm_kernels.selective_adam_update once per parameter
  group (submodules/clm_kernels/adam.cu:43-77); here every group is updated
  by one `tgs_selective_adam` launch with float4 accesses.
* SelectiveSophia: a Sophia step (Liu et al. 2023, "Sophia: A Scalable
  Stochastic Second-order Optimizer for Language Model Pre-training",
  Algorithm 3) with the same masked, one-launch structure. TideGS has no
  Sophia; the Hessian-diagonal estimate is the Hutchinson form
  u * (H u) with the diagonal Gauss-Newton proxy H = diag(g*g), i.e.
  h_hat = (u*g)^2 for u ~ N(0, 1), refreshed every k steps.
* ResidentAdamContext (optimizer.py:90-173): metadata only, unchanged.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence

import torch

from . import _lib


def _visibility_u8(visibility: torch.Tensor, device: torch.device) -> torch.Tensor:
    vis = visibility.reshape(-1)
    if vis.device != device:
        vis = vis.to(device)
    if vis.dtype != torch.bool:
        vis = vis != 0
    return vis.contiguous().view(torch.uint8)


def _launch_dense(name: str, groups: List[_lib.DenseGroup], vis: torch.Tensor, n_rows: int,
                  hessian_step: bool, device: torch.device) -> None:
    stream = _lib.stream_handle(device)
    for start in range(0, len(groups), _lib.MAX_GROUPS):
        chunk = groups[start:start + _lib.MAX_GROUPS]
        args = _lib.DenseArgs()
        for i, g in enumerate(chunk):
            args.groups[i] = g
        args.n_groups = len(chunk)
        args.visibility = vis.data_ptr()
        args.n_rows = int(n_rows)
        args.hessian_step = 1 if hessian_step else 0
        _lib.call(name, args, stream)


def _check_dense(param: torch.Tensor, others: Sequence[torch.Tensor], who: str) -> None:
    if param.device.type != "cuda":
        raise RuntimeError(f"{who} updates CUDA tensors only (tidegs_b200 has no CPU path)")
    for t in (param, *others):
        if t.dtype != torch.float32:
            raise RuntimeError(f"{who}: tensors must be float32, got {t.dtype}")
        if not t.is_contiguous():
            raise RuntimeError(f"{who}: tensors must be contiguous")
        if t.numel() != param.numel():
            raise RuntimeError(f"{who}: gradient/state shape does not match the parameter")


class SelectiveAdam(torch.optim.Adam):
    """Adam that updates only the rows whose visibility flag is set; no bias
    correction (the reference kernel has none). All groups in one launch."""

    def __init__(self, params, eps, betas):
        super().__init__(params=params, eps=eps, betas=betas)
        _lib.load()

    @torch.no_grad()
    def step(self, visibility):
        N = visibility.numel()
        launches = []
        device = None
        for group in self.param_groups:
            lr = group["lr"]
            eps = group["eps"]
            beta1, beta2 = group["betas"]
            assert len(group["params"]) == 1, "more than one tensor in group"
            param = group["params"][0]
            if param.grad is None:
                continue
            state = self.state[param]
            if len(state) == 0:
                state["step"] = torch.tensor(0.0, dtype=torch.float32)
                state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                state["exp_avg_sq"] = torch.zeros_like(param, memory_format=torch.preserve_format)
            exp_avg = state["exp_avg"]
            exp_avg_sq = state["exp_avg_sq"]
            if N == 0 or param.numel() == 0:
                continue
            M = param.numel() // N
            if M * N != param.numel():
                raise RuntimeError(
                    f"SelectiveAdam: parameter numel {param.numel()} is not a multiple of "
                    f"visibility numel {N}")
            grad = param.grad
            _check_dense(param, (grad, exp_avg, exp_avg_sq), "SelectiveAdam")
            if device is None:
                device = param.device
            elif param.device != device:
                raise RuntimeError("SelectiveAdam: all parameters must share one device")
            launches.append(_lib.DenseGroup(
                param=param.data_ptr(), grad=grad.data_ptr(), exp_avg=exp_avg.data_ptr(),
                exp_avg_sq=exp_avg_sq.data_ptr(), noise=None, width=M, lr=float(lr),
                beta1=float(beta1), beta2=float(beta2), eps=float(eps), rho=0.0,
                weight_decay=0.0))
        if not launches:
            return
        vis = _visibility_u8(visibility, device)
        _launch_dense("tgs_selective_adam", launches, vis, N, False, device)


class SelectiveSophia(torch.optim.Optimizer):
    """Masked Sophia: rows with visibility set get
        m = b1*m + (1-b1)*g
        every k-th step (t % k == 1): h = b2*h + (1-b2)*(u*g)^2, u ~ N(0,1)
        p = p - lr*wd*p                       (decoupled decay, off by default)
        p = p - lr * clip(m / max(rho*h, eps), 1)
    State per parameter: "step" (int), "exp_avg" (m), "hessian" (h).
    The noise u comes from `noise` (one tensor per parameter, in group order)
    or, when omitted, from this optimizer's seeded CUDA generator."""

    def __init__(self, params, lr=1e-4, betas=(0.965, 0.99), rho=0.04, eps=1e-15,
                 weight_decay=0.0, k=10, seed: int = 0):
        if k < 1:
            raise ValueError(f"SelectiveSophia: k must be >= 1, got {k}")
        defaults = dict(lr=lr, betas=betas, rho=rho, eps=eps, weight_decay=weight_decay, k=k)
        super().__init__(params, defaults)
        self._seed = int(seed)
        self._generators = {}
        _lib.load()

    def _noise_like(self, param: torch.Tensor) -> torch.Tensor:
        gen = self._generators.get(param.device)
        if gen is None:
            gen = torch.Generator(device=param.device).manual_seed(self._seed)
            self._generators[param.device] = gen
        return torch.randn(param.shape, generator=gen, device=param.device, dtype=torch.float32)

    @torch.no_grad()
    def step(self, visibility, noise: Optional[Sequence[torch.Tensor]] = None):
        N = visibility.numel()
        per_step = {}
        device = None
        noise_iter = iter(noise) if noise is not None else None
        keep = []
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            for param in group["params"]:
                u = next(noise_iter) if noise_iter is not None else None
                if param.grad is None:
                    continue
                state = self.state[param]
                if len(state) == 0:
                    state["step"] = 0
                    state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                    state["hessian"] = torch.zeros_like(param, memory_format=torch.preserve_format)
                state["step"] += 1
                t = state["step"]
                hess = (t % group["k"]) == (1 % group["k"])
                if N == 0 or param.numel() == 0:
                    continue
                M = param.numel() // N
                if M * N != param.numel():
                    raise RuntimeError(
                        f"SelectiveSophia: parameter numel {param.numel()} is not a multiple of "
                        f"visibility numel {N}")
                if hess:
                    if u is None:
                        u = self._noise_like(param)
                    u = u.to(device=param.device, dtype=torch.float32).contiguous()
                    keep.append(u)
                _check_dense(param, (param.grad, state["exp_avg"], state["hessian"])
                             + ((u,) if hess else ()), "SelectiveSophia")
                if device is None:
                    device = param.device
                elif param.device != device:
                    raise RuntimeError("SelectiveSophia: all parameters must share one device")
                per_step.setdefault(bool(hess), []).append(_lib.DenseGroup(
                    param=param.data_ptr(), grad=param.grad.data_ptr(),
                    exp_avg=state["exp_avg"].data_ptr(), exp_avg_sq=state["hessian"].data_ptr(),
                    noise=u.data_ptr() if hess else None, width=M, lr=float(group["lr"]),
                    beta1=float(beta1), beta2=float(beta2), eps=float(group["eps"]),
                    rho=float(group["rho"]), weight_decay=float(group["weight_decay"])))
        if not per_step:
            return
        vis = _visibility_u8(visibility, device)
        for hess, groups in per_step.items():
            _launch_dense("tgs_sophia_step", groups, vis, N, hess, device)
        del keep


class ResidentAdamContext:
    """Metadata context for the resident-block Adam updater: holds the single
    "unified_params" group, Adam hyperparameters and per-column learning rates
    that GPUResidentAdam reads. It performs no updates."""

    def __init__(self, params, columns_sizes, columns_lr, lr=1e-3, bias_correction=True,
                 betas=(0.9, 0.999), eps=1e-15, weight_decay=0, amsgrad=False, adamw_mode=False,
                 fp32_optimizer_states=True, fused=False, sparse=False):
        if len(params) != 1 or params[0].get("name") != "unified_params":
            raise RuntimeError(
                "ResidentAdamContext expects the single unified_params metadata group "
                "used by the Pure SSD/Tide release path."
            )
        group = dict(params[0])
        param_list = list(group.get("params", []))
        if len(param_list) != 1:
            raise RuntimeError("ResidentAdamContext expects one metadata tensor.")
        if param_list[0].is_cuda:
            raise AssertionError(
                "ResidentAdamContext metadata tensor must stay on CPU; resident "
                "blocks are materialized separately for GPUResidentAdam."
            )
        group["params"] = param_list
        group.setdefault("lr", lr)
        group.setdefault("bias_correction", bias_correction)
        group.setdefault("betas", betas)
        group.setdefault("eps", eps)
        group.setdefault("weight_decay", weight_decay)
        group.setdefault("amsgrad", amsgrad)
        group.setdefault("adamw_mode", adamw_mode)
        group.setdefault("fp32_optimizer_states", fp32_optimizer_states)
        self.param_groups = [group]
        self.state = {}
        self.columns_sizes = columns_sizes
        self.columns_lr = (torch.tensor(columns_lr, dtype=torch.float32)
                           if isinstance(columns_lr, list) else columns_lr)
        self.is_ssd_offload_mode = True
        self.cpu_adam = None
        self.gpu_adam = None
        self.fused = fused
        self.sparse = sparse

    def get_all_states(self):
        return []

    def zero_grad(self, set_to_none=False):
        for group in self.param_groups:
            for param in group.get("params", []):
                if param.grad is None:
                    continue
                if set_to_none:
                    param.grad = None
                else:
                    param.grad.zero_()

    def step(self, closure=None):
        if closure is not None:
            with torch.enable_grad():
                return closure()
        return None
