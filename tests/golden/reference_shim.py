"""Loads the reference TideGS hot-path modules on a CPU-only host, for golden
vector generation only (never imported at test or run time).

The reference modules are imported by file path under empty package stubs
(so storage/__init__.py and strategies/tide_engine/__init__.py, which pull in
the renderer and SSD stack, are not executed), CUDA streams/events/nvtx are
replaced by no-ops, and each module's `triton` is set to None so that the
reference's own torch fallback paths run.
"""
from __future__ import annotations

import contextlib
import importlib.util
import sys
import types
from pathlib import Path

import torch


class _NoOpStream:
    def __init__(self, *args, **kwargs):
        pass

    def wait_stream(self, other):
        pass

    def synchronize(self):
        pass

    def record_event(self, event=None):
        return event


class _NoOpEvent:
    def __init__(self, *args, **kwargs):
        pass

    def record(self, stream=None):
        pass

    def synchronize(self):
        pass

    def query(self):
        return True


def install_cuda_shims() -> None:
    torch.cuda.Stream = _NoOpStream
    torch.cuda.Event = _NoOpEvent
    torch.cuda.stream = lambda s=None: contextlib.nullcontext()
    torch.cuda.device = lambda d=None: contextlib.nullcontext()
    torch.cuda.current_stream = lambda device=None: _NoOpStream()
    torch.cuda.empty_cache = lambda: None
    torch.cuda.synchronize = lambda device=None: None
    torch.cuda.nvtx.range = lambda *a, **k: contextlib.nullcontext()


def _stub_package(name: str, path: Path) -> None:
    if name in sys.modules:
        return
    mod = types.ModuleType(name)
    mod.__path__ = [str(path)]
    sys.modules[name] = mod


def load_reference(root: Path):
    """Returns (block_reader, double_buffer_gpu, gpu_working_set,
    gpu_resident_optimizer) modules of the reference at `root`."""
    root = Path(root)
    install_cuda_shims()
    _stub_package("storage", root / "storage")
    _stub_package("strategies", root / "strategies")
    _stub_package("strategies.tide_engine", root / "strategies" / "tide_engine")

    def load(name: str, rel: str):
        if name in sys.modules and getattr(sys.modules[name], "__file__", None):
            return sys.modules[name]
        spec = importlib.util.spec_from_file_location(name, root / rel)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        if hasattr(mod, "triton"):
            mod.triton = None
        return mod

    load("storage.schedule_utils", "storage/schedule_utils.py")
    block_reader = load("storage.block_reader", "storage/block_reader.py")
    dbuf = load("strategies.tide_engine.double_buffer_gpu",
                "strategies/tide_engine/double_buffer_gpu.py")
    wset = load("strategies.tide_engine.gpu_working_set",
                "strategies/tide_engine/gpu_working_set.py")
    gro = load("strategies.tide_engine.gpu_resident_optimizer",
               "strategies/tide_engine/gpu_resident_optimizer.py")
    return block_reader, dbuf, wset, gro
