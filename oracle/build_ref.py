"""Builds the reference's SelectiveAdam kernel for B200 -- test infrastructure.

    python oracle/build_ref.py [--reference PATH]

Compiles submodules/clm_kernels/adam.cu of the reference tree, in place (it is
read, never copied), with oracle/ref_binding.cpp into the importable module
oracle/_ref/clm_adam_ref*.so for sm_100a, with the reference's own nvcc
flag (-O3, setup.py:27). The result is a checker for tests and a GPU
comparison point; nothing in tidegs_b200/ loads it. When the reference tree
is absent (as on the GPU box) nothing is built and the prebuilt module that
travelled with the repository is used.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
# the reference checkout beside this repository (override: TIDEGS_REFERENCE)
DEFAULT_REFERENCE = str(HERE.parent.parent / "reference")
MODULE = "clm_adam_ref"


def reference_root(explicit: str | None = None) -> Path | None:
    root = Path(explicit or os.environ.get("TIDEGS_REFERENCE", DEFAULT_REFERENCE))
    src = root / "submodules" / "clm_kernels" / "adam.cu"
    return root if src.exists() else None


def build(root: Path, verbose: bool = False):
    from torch.utils.cpp_extension import load

    OUT.mkdir(parents=True, exist_ok=True)
    kdir = root / "submodules" / "clm_kernels"
    return load(
        name=MODULE,
        sources=[str(kdir / "adam.cu"), str(HERE / "ref_binding.cpp")],
        extra_include_paths=[str(kdir)],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_cflags=["-O3"],
        build_directory=str(OUT),
        verbose=verbose,
    )


GSPLAT_MODULE = "gsplat_ref"
GSPLAT_OUT = OUT / "gsplat"
# the kernels of the engine's render path (projection, tile intersection,
# rasterization), compiled with gsplat's own nvcc flags (its setup.py:79-94)
GSPLAT_SOURCES = ("fully_fused_projection_fwd.cu", "fully_fused_projection_bwd.cu",
                  "isect_tiles.cu", "rasterize_to_pixels_fwd.cu", "rasterize_to_pixels_bwd.cu",
                  "compute_sh_fwd.cu", "compute_sh_bwd.cu")


def build_gsplat(root: Path, verbose: bool = False):
    """Compiles the reference's gsplat 1.0.0 render-path kernels (vendored
    sources, read in place) into oracle/_ref/gsplat/gsplat_ref*.so."""
    from torch.utils.cpp_extension import load

    csrc = root / "submodules" / "gsplat" / "gsplat" / "cuda" / "csrc"
    GSPLAT_OUT.mkdir(parents=True, exist_ok=True)
    return load(
        name=GSPLAT_MODULE,
        sources=[str(csrc / f) for f in GSPLAT_SOURCES] + [str(HERE / "gsplat_ref_binding.cpp")],
        extra_include_paths=[str(csrc), str(csrc / "third_party" / "glm")],
        extra_cuda_cflags=["-O3", "--use_fast_math", "--expt-relaxed-constexpr",
                           "-diag-suppress", "20012",
                           "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_cflags=["-O3", "-Wno-sign-compare"],
        build_directory=str(GSPLAT_OUT),
        verbose=verbose,
    )


def load_prebuilt_gsplat():
    """Imports the prebuilt reference gsplat module (None if absent)."""
    import importlib.util

    import torch  # noqa: F401

    for path in sorted(GSPLAT_OUT.glob(f"{GSPLAT_MODULE}*.so")):
        spec = importlib.util.spec_from_file_location(GSPLAT_MODULE, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod
    return None


def build_if_reference_present() -> bool:
    root = reference_root()
    if root is None:
        return False
    build(root)
    if (root / "submodules" / "gsplat" / "gsplat" / "cuda" / "csrc").exists():
        build_gsplat(root)
    return True


def load_prebuilt():
    """Imports the prebuilt module from oracle/_ref (None if absent)."""
    import importlib.util

    import torch  # noqa: F401  (loads the libraries the extension links against)

    for path in sorted(OUT.glob(f"{MODULE}*.so")):
        spec = importlib.util.spec_from_file_location(MODULE, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod
    return None


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=None)
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    root = reference_root(args.reference)
    if root is None:
        print("reference tree not found; nothing built")
        return 1
    build(root, verbose=args.verbose)
    build_gsplat(root, verbose=args.verbose)
    print("built into", OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
