"""ctypes binding of libtidegs_b200.so (declared in include/tidegs_b200.h).

The library is the only compute path of this package: there is no CPU or
torch fallback. If the shared library is missing, `load()` raises, and every
class that needs it raises at construction time.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path
from typing import Optional

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libtidegs_b200.so"
ABI_VERSION = 1
NUM_COMPONENTS = 6
ROW_WIDTH = 59
STATE_ROW_FLOATS = 128
MAX_GROUPS = 16
MAX_PEERS = 64
PEER_HANDLE_BYTES = 64

LAYOUT_CACHE = 0
LAYOUT_UNIFIED = 1

DEV_ERRORS = {
    1: "local row id out of range",
    2: "local row ids are not strictly ascending",
    3: "local row id is not inside any resident block",
    4: "bounded device wait timed out",
    5: "inconsistent copy plan",
    6: "filter id is not among the touched rows",
}

_vp = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f32 = C.c_float


class ResidentCountArgs(C.Structure):
    _fields_ = [
        ("pos_start", _vp), ("pos_end", _vp), ("pos_slot", _vp), ("n_positions", _i32),
        ("block_size", _i64), ("param_rows", _i64), ("local_ids", _vp), ("n_rows", _i64),
        ("slot_step", _vp), ("slot_stamp", _vp), ("slot_bias", _vp), ("step_table", _vp),
        ("step_table_len", _i32), ("n_slots", _i32), ("pos_count", _vp), ("err", _vp),
        ("chunk_table", _vp),
    ]


class ResidentAdamArgs(C.Structure):
    _fields_ = [
        ("param", _vp * NUM_COMPONENTS), ("grad", _vp * NUM_COMPONENTS),
        ("lr", _f32 * NUM_COMPONENTS), ("beta1", _f32), ("beta2", _f32), ("eps", _f32),
        ("one_minus_beta1", _f32), ("one_minus_beta2", _f32),
        ("batch_size", _f32), ("pos_start", _vp), ("pos_end", _vp), ("pos_slot", _vp),
        ("n_positions", _i32), ("block_size", _i64), ("local_ids", _vp), ("n_rows", _i64),
        ("state", _vp), ("slot_stamp", _vp), ("slot_bias", _vp), ("err", _vp),
        ("chunk_table", _vp),
    ]


class DenseGroup(C.Structure):
    _fields_ = [
        ("param", _vp), ("grad", _vp), ("exp_avg", _vp), ("exp_avg_sq", _vp), ("noise", _vp),
        ("width", _i64), ("lr", _f32), ("beta1", _f32), ("beta2", _f32), ("eps", _f32),
        ("rho", _f32), ("weight_decay", _f32),
    ]


class DenseArgs(C.Structure):
    _fields_ = [
        ("groups", DenseGroup * MAX_GROUPS), ("n_groups", _i32), ("visibility", _vp),
        ("n_rows", _i64), ("hessian_step", _i32),
    ]


class UnpackArgs(C.Structure):
    _fields_ = [
        ("packed", _vp), ("n_rows", _i64), ("layout", _i32), ("comp", _vp * NUM_COMPONENTS),
        ("target_offset", _i64), ("global_ids", _vp), ("block_ids", _vp), ("block_size", _i64),
        ("err", _vp), ("block_dst", _vp),
    ]


class CopyBlocksArgs(C.Structure):
    _fields_ = [
        ("src_comp", _vp * NUM_COMPONENTS), ("src_global_ids", _vp),
        ("dst_comp", _vp * NUM_COMPONENTS), ("dst_global_ids", _vp),
        ("src_start", _vp), ("dst_start", _vp), ("row_count", _vp), ("n_blocks", _i32),
        ("max_rows", _i64), ("err", _vp),
    ]


class PackArgs(C.Structure):
    _fields_ = [
        ("comp", _vp * NUM_COMPONENTS), ("src_start", _vp), ("row_count", _vp),
        ("out_start", _vp), ("n_plans", _i32), ("max_rows", _i64), ("out", _vp),
        ("layout", _i32), ("err", _vp),
    ]


class BlockSumArgs(C.Structure):
    _fields_ = [
        ("recv", _vp), ("n_recv_blocks", _i64), ("contrib_offsets", _vp),
        ("contrib_blocks", _vp), ("n_out", _i32), ("block_size", _i64),
        ("out", _vp * NUM_COMPONENTS), ("err", _vp),
    ]


class PeerHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * PEER_HANDLE_BYTES)]


class GradPushArgs(C.Structure):
    _fields_ = [
        ("comp", _vp * NUM_COMPONENTS), ("src_start", _vp), ("row_count", _vp),
        ("dst_rank", _vp), ("dst_row", _vp), ("n_tiles", _i32), ("max_rows", _i64),
        ("recv", _vp * MAX_PEERS), ("recv_rows", _i64 * MAX_PEERS), ("n_ranks", _i32),
        ("err", _vp),
    ]


class ResidentAdamSumArgs(C.Structure):
    _fields_ = [
        ("adam", ResidentAdamArgs), ("grad_src", _vp), ("grad_rows", _vp), ("n_ranks", _i32),
        ("seg_begin", _vp), ("n_segments", _i32), ("contrib_offsets", _vp),
        ("contrib_rank", _vp), ("contrib_row", _vp), ("rotate_rows", _i64), ("err", _vp),
        ("max_ctas", _i32),
    ]


class SparseAccumArgs(C.Structure):
    _fields_ = [
        ("touched", _vp), ("n_touched", _i64), ("pos_map", _vp), ("pos_map_len", _i64),
        ("filter", _vp), ("n_filter", _i64),
        ("src", _vp * NUM_COMPONENTS), ("src_stride", _i64 * NUM_COMPONENTS),
        ("acc", _vp * NUM_COMPONENTS), ("unique_filter", _i32), ("err", _vp),
    ]


class CullArgs(C.Structure):
    _fields_ = [
        ("centers", _vp), ("radii", _vp), ("n_blocks", _i64), ("subset", _vp), ("n_items", _i64),
        ("planes", _vp), ("n_cameras", _i32), ("out_ids", _vp), ("out_stride", _i64),
        ("out_counts", _vp), ("slice_counts", _vp), ("err", _vp),
    ]


class ProjectArgs(C.Structure):
    _fields_ = [
        ("means", _vp), ("quats", _vp), ("scales", _vp), ("viewmats", _vp), ("Ks", _vp),
        ("n_cameras", _i32), ("n_gaussians", _i64), ("image_width", _i32),
        ("image_height", _i32), ("eps2d", C.c_float), ("near_plane", C.c_float),
        ("far_plane", C.c_float), ("radius_clip", C.c_float), ("radii", _vp), ("means2d", _vp),
        ("depths", _vp), ("conics", _vp), ("compensations", _vp),
    ]


class ProjectBwdArgs(C.Structure):
    _fields_ = [
        ("fwd", ProjectArgs), ("v_means2d", _vp), ("v_depths", _vp), ("v_conics", _vp),
        ("v_compensations", _vp), ("v_means", _vp), ("v_quats", _vp), ("v_scales", _vp),
    ]


class RasterArgs(C.Structure):
    _fields_ = [
        ("means2d", _vp), ("conics", _vp), ("colors", _vp), ("opacities", _vp),
        ("backgrounds", _vp), ("n_cameras", _i32), ("n_gaussians", _i64), ("channels", _i32),
        ("image_width", _i32), ("image_height", _i32), ("tile_size", _i32),
        ("tile_width", _i32), ("tile_height", _i32), ("tile_offsets", _vp),
        ("flatten_ids", _vp), ("n_isects", _i64), ("render_colors", _vp),
        ("render_alphas", _vp), ("last_ids", _vp),
    ]


class RasterBwdArgs(C.Structure):
    _fields_ = [
        ("fwd", RasterArgs), ("v_render_colors", _vp), ("v_render_alphas", _vp),
        ("v_means2d_abs", _vp), ("v_means2d", _vp), ("v_conics", _vp), ("v_colors", _vp),
        ("v_opacities", _vp),
    ]


class ShArgs(C.Structure):
    _fields_ = [("dirs", _vp), ("coeffs", _vp), ("masks", _vp), ("n", _i64), ("K", _i32),
                ("degree", _i32), ("colors", _vp)]


class ShBwdArgs(C.Structure):
    _fields_ = [("fwd", ShArgs), ("v_colors", _vp), ("v_coeffs", _vp), ("v_dirs", _vp)]


# name -> (restype, argtypes). Keep in sync with include/tidegs_b200.h.
SIGNATURES = {
    "tgs_version": (C.c_int, []),
    "tgs_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "tgs_resident_adam_count": (C.c_int, [C.POINTER(ResidentCountArgs), _vp]),
    "tgs_resident_adam_apply": (C.c_int, [C.POINTER(ResidentAdamArgs), _vp]),
    "tgs_selective_adam": (C.c_int, [C.POINTER(DenseArgs), _vp]),
    "tgs_sophia_step": (C.c_int, [C.POINTER(DenseArgs), _vp]),
    "tgs_unpack_rows": (C.c_int, [C.POINTER(UnpackArgs), _vp]),
    "tgs_copy_blocks": (C.c_int, [C.POINTER(CopyBlocksArgs), _vp]),
    "tgs_fill_global_ids": (C.c_int, [_vp, _i64, _vp, _i64, _i64, _vp]),
    "tgs_build_block_starts": (C.c_int, [_vp, _i64, _vp, _vp, _i64, _vp]),
    "tgs_global_to_local": (C.c_int, [_vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "tgs_compact_scratch_words": (_i64, [_i64]),
    "tgs_global_to_local_compact": (C.c_int, [_vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "tgs_global_to_local_compact_noalloc": (C.c_int, [_vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "tgs_h2d_blocks": (C.c_int, [C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_i64), _i32, _vp]),
    "tgs_d2h_blocks": (C.c_int, [C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_i64), _i32, _vp]),
    "tgs_dirty_mark": (C.c_int, [_vp, _i64, _vp, _i64, _i32, _vp]),
    "tgs_dirty_select": (C.c_int, [_vp, _i64, _vp, _i64, _vp, _vp, _vp]),
    "tgs_dirty_list": (C.c_int, [_vp, _i64, _vp, _vp, _vp]),
    "tgs_pack_rows": (C.c_int, [C.POINTER(PackArgs), _vp]),
    "tgs_block_bounds": (C.c_int, [_vp, _vp, _vp, _i32, _vp, _vp]),
    "tgs_block_grad_sum": (C.c_int, [C.POINTER(BlockSumArgs), _vp]),
    "tgs_copy_small": (C.c_int, [_vp, _vp, _i64, _vp]),
    "tgs_grad_push": (C.c_int, [C.POINTER(GradPushArgs), _vp]),
    "tgs_peer_buffer_alloc": (C.c_int, [_i64, C.POINTER(_vp), C.POINTER(PeerHandle)]),
    "tgs_peer_buffer_free": (C.c_int, [_vp]),
    "tgs_peer_buffer_open": (C.c_int, [C.POINTER(PeerHandle), C.POINTER(_vp)]),
    "tgs_peer_buffer_close": (C.c_int, [_vp]),
    "tgs_peer_export": (C.c_int, [_vp, C.POINTER(PeerHandle), C.POINTER(_i64)]),
    "tgs_peer_access_enable": (C.c_int, [_i32]),
    "tgs_resident_adam_apply_sum": (C.c_int, [C.POINTER(ResidentAdamSumArgs), _vp]),
    "tgs_bitmap_set": (C.c_int, [_vp, _i64, _vp, _i64, _vp, _vp]),
    "tgs_bitmap_list_scratch_words": (_i64, [_i64]),
    "tgs_bitmap_list": (C.c_int, [_vp, _i64, _vp, _vp, _vp, _vp, _vp]),
    "tgs_gather_i64": (C.c_int, [_vp, _vp, _i64, _vp, _i64, _vp, _vp]),
    "tgs_sparse_grad_accumulate": (C.c_int, [C.POINTER(SparseAccumArgs), _vp]),
    "tgs_block_spheres": (C.c_int, [_vp, _i64, _vp, _vp, _vp]),
    "tgs_frustum_cull": (C.c_int, [C.POINTER(CullArgs), _vp]),
    "tgs_frustum_cull_slices": (_i64, [_i64]),
    "tgs_project_fwd": (C.c_int, [C.POINTER(ProjectArgs), _vp]),
    "tgs_project_bwd": (C.c_int, [C.POINTER(ProjectBwdArgs), _vp]),
    "tgs_isect_count": (C.c_int, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp]),
    "tgs_isect_tile_bits": (_i32, [_i32]),
    "tgs_isect_write": (C.c_int, [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                                  _vp]),
    "tgs_isect_depth_order_scratch_bytes": (C.c_int, [_i64, C.POINTER(C.c_size_t)]),
    "tgs_isect_key_bytes": (_i32, [_i32, _i32, _i32]),
    "tgs_isect_depth_order": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, C.c_size_t, _vp]),
    "tgs_isect_write_ordered": (C.c_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp,
                                          _vp, _vp, _vp]),
    "tgs_isect_sort_tiles_scratch_bytes": (C.c_int, [_i64, _i32, _i32, _i32,
                                                     C.POINTER(C.c_size_t)]),
    "tgs_isect_sort_tiles": (C.c_int, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                                       C.c_size_t, _vp]),
    "tgs_isect_expand_ids": (C.c_int, [_vp, _i32, _vp, _vp, _i64, _vp, _vp]),
    "tgs_isect_offsets": (C.c_int, [_vp, _i64, _i32, _i32, _i32, _vp, _vp]),
    "tgs_rasterize_fwd": (C.c_int, [C.POINTER(RasterArgs), _vp]),
    "tgs_rasterize_bwd": (C.c_int, [C.POINTER(RasterBwdArgs), _vp]),
    "tgs_sh_fwd": (C.c_int, [C.POINTER(ShArgs), _vp]),
    "tgs_sh_bwd": (C.c_int, [C.POINTER(ShBwdArgs), _vp]),
}

_lock = threading.Lock()
_lib: Optional[C.CDLL] = None


def load() -> C.CDLL:
    """Loads the CUDA library (once). Raises RuntimeError when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("TIDEGS_B200_LIB", str(LIB_PATH)))
        if not path.exists():
            raise RuntimeError(
                f"tidegs_b200 CUDA library not found at {path}; build it with "
                "`python -m tidegs_b200.build` (there is no CPU fallback)"
            )
        lib = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        ver = lib.tgs_version()
        if ver != ABI_VERSION:
            raise RuntimeError(f"tidegs_b200 ABI mismatch: library {ver}, bindings {ABI_VERSION}")
        _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(1024)
    lib.tgs_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


# Kernels each entry point launches when it has work (for launch accounting).
KERNELS_PER_CALL = {
    "tgs_resident_adam_count": 2, "tgs_resident_adam_apply": 1, "tgs_selective_adam": 1,
    "tgs_sophia_step": 1, "tgs_unpack_rows": 1, "tgs_copy_blocks": 1, "tgs_fill_global_ids": 1,
    "tgs_build_block_starts": 1, "tgs_global_to_local": 1, "tgs_global_to_local_compact": 3,
    "tgs_global_to_local_compact_noalloc": 3,
    "tgs_dirty_mark": 1, "tgs_dirty_select": 1, "tgs_dirty_list": 1, "tgs_pack_rows": 1,
    "tgs_block_bounds": 1, "tgs_block_grad_sum": 1, "tgs_copy_small": 1, "tgs_grad_push": 1,
    "tgs_resident_adam_apply_sum": 1, "tgs_bitmap_list": 3, "tgs_gather_i64": 1, "tgs_bitmap_set": 1,
    "tgs_sparse_grad_accumulate": 1, "tgs_block_spheres": 1, "tgs_frustum_cull": 2,
    "tgs_project_fwd": 1, "tgs_project_bwd": 1, "tgs_isect_count": 1, "tgs_isect_write": 1,
    "tgs_isect_offsets": 1, "tgs_rasterize_fwd": 1, "tgs_rasterize_bwd": 1,
    "tgs_isect_write_ordered": 1, "tgs_isect_expand_ids": 1, "tgs_sh_fwd": 1, "tgs_sh_bwd": 1,
    # iota + the library radix sort and scan (their kernel counts depend on
    # the library version and are not counted here)
    "tgs_isect_depth_order": 1, "tgs_isect_sort_tiles": 0,
}
launch_counter = {"kernels": 0}


# TIDEGS_NVTX=1: every entry point call is an NVTX range named after it (for
# Nsight timelines; off by default, a push/pop costs about a microsecond).
NVTX = os.environ.get("TIDEGS_NVTX", "0") not in ("", "0")


def call(name: str, *args) -> None:
    """Calls entry point `name`; raises RuntimeError with the library message."""
    lib = load()
    if NVTX:
        torch.cuda.nvtx.range_push(name)
        try:
            status = getattr(lib, name)(*args)
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        status = getattr(lib, name)(*args)
    if status != 0:
        raise RuntimeError(f"[tidegs_b200] {name} failed (status {status}): {last_error()}")
    launch_counter["kernels"] += KERNELS_PER_CALL.get(name, 0)


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device, stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def require_cuda(device, who: str) -> torch.device:
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError(
            f"{who} runs only on CUDA devices (got {device}); tidegs_b200 has no CPU path"
        )
    if not torch.cuda.is_available():
        raise RuntimeError(f"{who}: CUDA is not available")
    load()
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def decode_device_error(err_host) -> Optional[str]:
    """err_host: 4 ints read back from a device error word."""
    code = int(err_host[0])
    if code == 0:
        return None
    index = (int(err_host[1]) & 0xFFFFFFFF) | ((int(err_host[2]) & 0xFFFFFFFF) << 32)
    return f"{DEV_ERRORS.get(code, f'device error {code}')} (index {index}, aux {int(err_host[3])})"
