"""Touched-only gradient accumulation of a camera batch.

Drop-in for the part of the training step that builds the resident
optimizer's sparse input (strategies/tide_engine/engine.py:1793-1826) and
fills it camera by camera (:2434-2471). The reference marks the union of the
cameras' local filters in a bool mask (`scatter_`), lists it with `nonzero`,
gathers `local_to_global` for it, zero-fills six compact gradient tensors,
and for every camera runs `searchsorted` plus six `scatter_add_` launches.
Here: one bitmap-set launch per camera, one ordered bitmap compaction, one
gather, and one launch per camera for all six components.

    acc = SparseGradAccumulator(filters_local, num_rows, local_to_global)
    for cam, filt in enumerate(filters_local):        # the micro-batch loop
        ...                                            # render + backward
        acc.add(filt, xyz.grad, opacity.grad, scaling.grad, rotation.grad, shs.grad)
    acc.check()
    optimizer.step(iteration, gaussians, acc.sparse_grad_local_ids,
                   acc.sparse_grad_components)

Additions land in camera order, one rounding each, so the compact gradients
equal the reference's sequential `scatter_add_` results bit for bit when no
id repeats inside one filter (projection filters never repeat an id).
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch

from . import _lib, _ops


class SparseGradAccumulator:
    def __init__(self, filters_local: Sequence[Optional[torch.Tensor]], num_rows: int,
                 local_to_global: Optional[torch.Tensor] = None, device=None):
        if device is None:
            device = next((f.device for f in filters_local if f is not None and f.numel()),
                          torch.device("cuda", torch.cuda.current_device()))
        self.device = _lib.require_cuda(device, "SparseGradAccumulator")
        self.num_rows = int(num_rows)
        self._err = torch.zeros(4, dtype=torch.int32, device=self.device)
        stream = _lib.stream_handle(self.device)
        bitmap = torch.zeros(_ops.bitmap_words(self.num_rows), dtype=torch.int32,
                             device=self.device)
        total = 0
        keep = []
        for f in filters_local:
            if f is None or f.numel() == 0:
                continue
            f = f.to(device=self.device, dtype=torch.int64).contiguous()
            keep.append(f)
            _lib.call("tgs_bitmap_set", bitmap.data_ptr(), self.num_rows, f.data_ptr(), f.numel(),
                      self._err.data_ptr(), stream)
            total += f.numel()
        cap = min(self.num_rows, total)
        out = torch.zeros(cap + 1, dtype=torch.int64, device=self.device)
        # row -> position in the touched list (-1: untouched), for one-load
        # lookups in add() (int32: fewer than 2^31 touched rows)
        self._pos_map = None
        if cap:
            if cap < 2 ** 31:
                self._pos_map = torch.full((self.num_rows,), -1, dtype=torch.int32,
                                           device=self.device)
            scratch = torch.empty(int(_lib.load().tgs_bitmap_list_scratch_words(self.num_rows)),
                                  dtype=torch.int64, device=self.device)
            _lib.call("tgs_bitmap_list", bitmap.data_ptr(), self.num_rows, out[1:].data_ptr(),
                      out[:1].data_ptr(), scratch.data_ptr(), _lib.ptr(self._pos_map), stream)
        n = int(out[0].item())  # the touched count (the reference reads it too)
        self._raise_on_error("filter ids")
        del keep, bitmap
        #: ascending local ids of every row some camera of the batch sees
        self.sparse_grad_local_ids = out[1:1 + n]
        #: their global ids on the host, or None without a local_to_global map
        self.sparse_visibility_indices = None
        if local_to_global is not None:
            l2g = local_to_global.to(device=self.device, dtype=torch.int64).contiguous()
            vis = torch.empty(n, dtype=torch.int64, device=self.device)
            _lib.call("tgs_gather_i64", vis.data_ptr(), l2g.data_ptr(), l2g.numel(),
                      self.sparse_grad_local_ids.data_ptr(), n, self._err.data_ptr(), stream)
            self.sparse_visibility_indices = vis.cpu()
            self._raise_on_error("local_to_global")
        #: compact gradients [touched, W] of the six components
        self.sparse_grad_components: Dict[str, torch.Tensor] = {
            name: torch.zeros((n, w), dtype=torch.float32, device=self.device)
            for name, w in _ops.WIDTHS.items()}

    @property
    def touched_count(self) -> int:
        return int(self.sparse_grad_local_ids.numel())

    def add(self, filter_local: torch.Tensor, xyz_grad: torch.Tensor, opacity_grad: torch.Tensor,
            scaling_grad: torch.Tensor, rotation_grad: torch.Tensor,
            shs_grad: Optional[torch.Tensor] = None, unique_filter: bool = True) -> None:
        """Adds one camera's gradients (rows in filter order). shs_grad is
        the [n, 48] SH gradient (dc = columns 0..2, rest = 3..47) or None,
        as in the reference. unique_filter=False accumulates with atomics
        (ids may repeat; order of repeats unspecified)."""
        n = int(filter_local.numel())
        if n == 0:
            return
        f = filter_local.to(device=self.device, dtype=torch.int64).contiguous()
        srcs = [xyz_grad, opacity_grad, scaling_grad, rotation_grad]
        if shs_grad is not None:
            if shs_grad.dim() != 2 or shs_grad.shape[1] < 48:
                raise ValueError("SparseGradAccumulator.add: shs_grad must be [n, 48]")
            srcs += [shs_grad[:, 0:3], shs_grad[:, 3:48]]
        else:
            srcs += [None, None]
        args = _lib.SparseAccumArgs()
        args.touched = self.sparse_grad_local_ids.data_ptr()
        args.n_touched = self.touched_count
        args.pos_map = _lib.ptr(self._pos_map)
        args.pos_map_len = self.num_rows if self._pos_map is not None else 0
        args.filter = f.data_ptr()
        args.n_filter = n
        for c, (name, t) in enumerate(zip(_ops.COMPONENTS, srcs)):
            acc = self.sparse_grad_components[name]
            args.acc[c] = acc.data_ptr()
            if t is None:
                args.src[c] = None
                args.src_stride[c] = _ops.WIDTHS[name]
                continue
            w = _ops.WIDTHS[name]
            if (t.dtype != torch.float32 or t.device != self.device or t.dim() != 2
                    or t.shape[0] != n or t.shape[1] != w or t.stride(1) != 1):
                raise RuntimeError(f"SparseGradAccumulator.add: {name} gradient must be float32 "
                                   f"[{n}, {w}] rows with unit column stride on {self.device}")
            args.src[c] = t.data_ptr()
            args.src_stride[c] = t.stride(0)
        args.unique_filter = 1 if unique_filter else 0
        args.err = self._err.data_ptr()
        stream = torch.cuda.current_stream(self.device)
        _lib.call("tgs_sparse_grad_accumulate", args, stream.cuda_stream)
        f.record_stream(stream)

    def check(self) -> None:
        """Raises if an earlier add saw a filter id outside the touched rows."""
        self._raise_on_error("filter")

    def _raise_on_error(self, what: str) -> None:
        problem = _lib.decode_device_error(self._err.cpu().tolist())
        if problem is not None:
            raise RuntimeError(f"[SparseGradAccumulator] invalid {what}: {problem}")
