"""Block frustum culling with device-resident block spheres
(storage/gaussian_block.py:145-531 FrustumCuller, 6-plane path).

`BlockCuller` keeps the block bounds, sphere centers and radii in device
memory (the write-back's bounds kernel output can update them without a host
round trip) and culls any number of cameras in one launch of
`tgs_frustum_cull`, one CTA per camera. Only the 6x4 planes of each camera
are computed on the host (Gribb & Hartmann extraction, as the reference).
The visible sets equal the reference's numpy evaluation exactly: the kernels
round every float32 operation once in the reference's order.

Not provided: the legacy cone test (`use_6plane=False`, not the reference's
default); calling it raises NotImplementedError.
"""
from __future__ import annotations

import ctypes as C
import threading
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib, _ops

__all__ = ["BlockCuller", "extract_frustum_planes"]

_OPENCV_TO_OPENGL = np.diag(np.array([1, -1, -1, 1], dtype=np.float32))


def extract_frustum_planes(view_matrix: np.ndarray, proj_matrix: np.ndarray,
                           coordinate_system: str = "opengl", validate: bool = True) -> np.ndarray:
    """(6, 4) float32 normalized planes (left, right, bottom, top, near, far)
    of the view-projection matrix by the Gribb & Hartmann row sums, each
    scaled by 1/|(A, B, C)| (gaussian_block.py:145-228)."""
    view = np.asarray(view_matrix).copy()
    if coordinate_system == "opencv":
        view = _OPENCV_TO_OPENGL @ view
    vp = np.asarray(proj_matrix) @ view
    planes = np.zeros((6, 4), dtype=np.float32)
    for k in range(3):
        planes[2 * k] = vp[3, :] + vp[k, :]
        planes[2 * k + 1] = vp[3, :] - vp[k, :]
    # per plane with float32 scalars, the reference's evaluation (a vectorized
    # square may round differently from the scalar power)
    for i in range(6):
        norm = np.sqrt(planes[i, 0] ** 2 + planes[i, 1] ** 2 + planes[i, 2] ** 2)
        if not norm > 1e-8:
            raise ValueError(f"Degenerate frustum plane {i}: normal length = {norm}")
        planes[i] /= norm
    if validate and coordinate_system == "opengl" and (planes[4, 2] > 0 or planes[5, 2] < 0):
        import warnings

        warnings.warn(
            f"Suspicious plane orientations: near_z={planes[4, 2]:.3f}, "
            f"far_z={planes[5, 2]:.3f}. Expected near_z < 0 and far_z > 0 for OpenGL. "
            "Check projection matrix.")
    return planes


class BlockCuller:
    """FrustumCuller with the blocks' bounding spheres on the device
    (gaussian_block.py:264-531): same constructor, `update_block_bounds`,
    `cull`, `cull_subset`, `get_visibility_order`, plus `cull_cameras` for a
    whole camera batch in one launch."""

    def __init__(self, block_bounds, scene_radius: Optional[float] = None, block_size: int = 4096,
                 verbose: bool = True, device="cuda"):
        self.device = _lib.require_cuda(device, "FrustumCuller")
        self.scene_radius = scene_radius
        self.block_size = block_size
        self.verbose = bool(verbose)
        self._bounds_lock = threading.RLock()
        if isinstance(block_bounds, torch.Tensor):
            bounds = block_bounds.detach().to(self.device, torch.float32).contiguous().clone()
        else:
            bounds = torch.from_numpy(np.ascontiguousarray(block_bounds, dtype=np.float32)).to(
                self.device)
        if bounds.dim() != 2 or bounds.shape[1] != 6:
            raise ValueError(f"block_bounds must be (N, 6); got {tuple(bounds.shape)}")
        self.block_bounds = bounds
        self.num_blocks = int(bounds.shape[0])
        self.block_centers = torch.empty((self.num_blocks, 3), dtype=torch.float32,
                                         device=self.device)
        self.block_radii = torch.empty(self.num_blocks, dtype=torch.float32, device=self.device)
        self._err = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._spheres(self.block_bounds, self.block_centers, self.block_radii)
        half = (self.block_radii / np.float32(1.15)).cpu().numpy()  # logging statistics only
        radii = self.block_radii.cpu().numpy()
        self.block_radius = float(radii.max()) if radii.size else 0.0
        self.block_radius_min = float(half.min()) if half.size else 0.0
        self.block_radius_max = float(half.max()) if half.size else 0.0
        self.block_radius_median = float(np.median(half)) if half.size else 0.0
        self._log(f"[FrustumCuller-GPU] Initialized with {self.num_blocks} blocks")

    def _log(self, message: str) -> None:
        if self.verbose:
            print(message)

    def _spheres(self, bounds: torch.Tensor, centers: torch.Tensor, radii: torch.Tensor) -> None:
        _lib.call("tgs_block_spheres", bounds.data_ptr(), int(bounds.shape[0]), centers.data_ptr(),
                  radii.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)

    def update_block_bounds(self, block_ids, block_bounds) -> int:
        """Replaces the bounds of the listed blocks and their spheres
        (gaussian_block.py:318-340); `block_bounds` may be a device tensor
        (e.g. the write-back's bounds) or a host array."""
        ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
        if ids.size == 0:
            return 0
        if isinstance(block_bounds, torch.Tensor):
            bounds = block_bounds.detach().to(self.device, torch.float32).contiguous()
        else:
            bounds = torch.from_numpy(np.ascontiguousarray(block_bounds, dtype=np.float32)).to(
                self.device)
        if tuple(bounds.shape) != (ids.size, 6):
            raise ValueError(f"Expected block_bounds shape {(ids.size, 6)}, got "
                             f"{tuple(bounds.shape)}")
        if np.any(ids < 0) or np.any(ids >= self.num_blocks):
            raise IndexError("block_ids contains an out-of-range block")
        centers = torch.empty((ids.size, 3), dtype=torch.float32, device=self.device)
        radii = torch.empty(ids.size, dtype=torch.float32, device=self.device)
        self._spheres(bounds, centers, radii)
        idx = _ops.i64_to_device(ids, self.device)
        with self._bounds_lock:
            self.block_bounds.index_copy_(0, idx, bounds)
            self.block_centers.index_copy_(0, idx, centers)
            self.block_radii.index_copy_(0, idx, radii)
            self.block_radius = max(self.block_radius, float(radii.max().item()))
        return int(ids.size)

    # -- culling -------------------------------------------------------------
    def cull_cameras(self, cameras: Sequence[Tuple[np.ndarray, np.ndarray]], block_ids=None,
                     as_tensors: bool = False, planes: Optional[np.ndarray] = None):
        """Visible blocks of every (view_matrix, projection_matrix) in one
        launch: a list of ascending id lists (candidate order with
        `block_ids`), or with `as_tensors` the device tensors (ids
        [cameras, candidates], counts [cameras]). `planes` ([cameras, 6, 4]
        float32, from extract_frustum_planes) skips the host extraction for
        cameras whose planes the caller keeps; `cameras` is then unused."""
        if planes is None:
            planes = np.stack([extract_frustum_planes(v, p) for v, p in cameras]) \
                if len(cameras) else np.zeros((0, 6, 4), np.float32)
        planes = np.ascontiguousarray(planes, dtype=np.float32)
        n_cam = int(planes.shape[0])
        if n_cam == 0:
            return (torch.empty((0, 0), dtype=torch.int64, device=self.device),
                    torch.empty(0, dtype=torch.int64, device=self.device)) if as_tensors else []
        subset = None
        if block_ids is not None:
            ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
            if np.any(ids < 0) or np.any(ids >= self.num_blocks):
                raise ValueError("block_ids contains an out-of-range block")
            subset = _ops.i64_to_device(ids, self.device)
            n_items = int(ids.size)
        else:
            n_items = self.num_blocks
        planes_dev = torch.empty((n_cam, 6, 4), dtype=torch.float32, device=self.device)
        _ops.upload_into(planes_dev, planes)
        out = torch.empty((n_cam, max(1, n_items)), dtype=torch.int64, device=self.device)
        counts = torch.empty(n_cam, dtype=torch.int64, device=self.device)
        n_slices = int(_lib.load().tgs_frustum_cull_slices(n_items))
        slice_counts = torch.empty((n_cam, n_slices), dtype=torch.int64, device=self.device)
        stream = torch.cuda.current_stream(self.device)
        with self._bounds_lock:
            for c0 in range(0, n_cam, 65535):
                c1 = min(n_cam, c0 + 65535)
                args = _lib.CullArgs(self.block_centers.data_ptr(), self.block_radii.data_ptr(),
                                 self.num_blocks, subset.data_ptr() if subset is not None else None,
                                 n_items, planes_dev[c0].data_ptr(), c1 - c0, out[c0].data_ptr(),
                                 out.shape[1], counts[c0:].data_ptr(),
                                 slice_counts[c0].data_ptr(), self._err.data_ptr())
                _lib.call("tgs_frustum_cull", C.byref(args), stream.cuda_stream)
        if as_tensors:
            return out, counts
        host_counts = counts.cpu().numpy()
        host_ids = out.cpu().numpy()
        self._check()
        return [host_ids[c, :host_counts[c]].tolist() for c in range(n_cam)]

    def _check(self) -> None:
        code = int(self._err[0].item())
        if code:
            self._err.zero_()
            raise RuntimeError(f"[FrustumCuller] {_lib.DEV_ERRORS.get(code, code)}")

    def cull(self, camera_position: np.ndarray, view_matrix: np.ndarray,
             projection_matrix: np.ndarray, margin: float = 1.0,
             use_6plane: bool = True) -> List[int]:
        """Ascending ids of the blocks whose sphere is inside all six planes
        (gaussian_block.py:342-357, 429-465)."""
        if not use_6plane:
            raise NotImplementedError("the legacy cone test (use_6plane=False) is not provided")
        return self.cull_cameras([(view_matrix, projection_matrix)])[0]

    def cull_subset(self, camera_position: np.ndarray, view_matrix: np.ndarray,
                    projection_matrix: np.ndarray, block_ids, margin: float = 1.0,
                    use_6plane: bool = True) -> List[int]:
        """The visible ones among `block_ids`, in their order (a set is sorted
        first) (gaussian_block.py:359-406)."""
        if not use_6plane:
            raise NotImplementedError("the legacy cone test (use_6plane=False) is not provided")
        if isinstance(block_ids, set):
            block_ids = sorted(block_ids)
        ids = np.asarray(block_ids, dtype=np.int64).reshape(-1)
        if ids.size == 0:
            return []
        return self.cull_cameras([(view_matrix, projection_matrix)], block_ids=ids)[0]

    def get_visibility_order(self, visible_blocks: List[int],
                             camera_position: np.ndarray) -> List[int]:
        """Visible blocks front to back by squared center distance
        (gaussian_block.py:513-531; numpy argsort on the host over the
        device centers)."""
        if not visible_blocks:
            return []
        with self._bounds_lock:
            idx = _ops.i64_to_device(np.asarray(visible_blocks, dtype=np.int64), self.device)
            centers = self.block_centers.index_select(0, idx).cpu().numpy()
        diff = centers - camera_position
        order = np.argsort(np.sum(diff ** 2, axis=1))
        return [visible_blocks[i] for i in order]
