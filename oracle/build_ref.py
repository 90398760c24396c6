"""Builds the reference's kernels for B200 -- test infrastructure.

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


# ---------------------------------------------------------------------------
# The reference's Triton kernels of the hot path, compiled ahead of time for
# sm_100 from the reference's own sources (loaded by path; nothing is
# copied), so that the GPU box -- which has no reference tree -- can run them
# beside this library's kernels. Only the binary and Triton's metadata are
# kept, with the launch signature; tests/probes.py --ref-kernels loads them.
# ---------------------------------------------------------------------------
TRITON_OUT = OUT / "triton"


def _triton_jobs(dbuf, wset, gro):
    """(name, jit function, [(arg, type)], constexprs, num_warps) for each
    specialization, as the reference's launches at the benchmark's shapes
    get them (gpu_resident_optimizer.py:397-418, double_buffer_gpu.py:
    849-871, 952-961, 1066-1080, gpu_working_set.py:953-967, 1039-1046)."""
    f32p, i64p = "*fp32", "*i64"
    comps = ["xyz", "scaling", "rotation", "opacity", "features_dc", "features_rest"]
    adam = [("param_ptr", f32p), ("grad_ptr", f32p), ("exp_avg_ptr", f32p),
            ("exp_avg_sq_ptr", f32p), ("local_rows_ptr", i64p), ("state_rows_ptr", i64p),
            ("state_slots_ptr", i64p), ("bias_correction1_ptr", f32p),
            ("denom_scale_ptr", f32p), ("n_rows", "i32"), ("learning_rate", "fp32"),
            ("beta1", "fp32"), ("beta2", "fp32"), ("eps", "fp32"), ("batch_size", "fp32"),
            ("WIDTH", "constexpr"), ("BLOCK_SIZE", "constexpr")]
    jobs = [(f"fused_resident_adam_w{w}", gro._fused_resident_adam_kernel, adam,
             {"WIDTH": w, "BLOCK_SIZE": 256}, 4) for w in (1, 3, 4, 45)]
    unpack = ([("source", f32p)] + [(f"target_{c}", f32p) for c in comps]
              + [("target_offset", "i32"), ("num_rows", "i32"),
                 ("SOURCE_UNIFIED", "constexpr"), ("COPY_BLOCK_SIZE", "constexpr")])
    jobs.append(("unpack_streamed_rows_cache", dbuf._unpack_streamed_rows_kernel, unpack,
                 {"SOURCE_UNIFIED": False, "COPY_BLOCK_SIZE": 256}, 4))
    copy = ([(f"source_{c}", f32p) for c in comps] + [("source_global_ids", i64p),
            ("source_starts", i64p), ("target_starts", i64p)]
            + [(f"target_{c}", f32p) for c in comps] + [("target_global_ids", i64p),
            ("num_rows", "i32"), ("BLOCK_ROWS", "constexpr"), ("COPY_BLOCK_SIZE", "constexpr")])
    jobs.append(("copy_resident_rows_b16384", dbuf._copy_resident_rows_kernel, copy,
                 {"BLOCK_ROWS": 16384, "COPY_BLOCK_SIZE": 256}, 4))
    fill = [("block_ids", i64p), ("target_global_ids", i64p), ("target_offset", "i32"),
            ("num_rows", "i32"), ("BLOCK_ROWS", "constexpr"), ("COPY_BLOCK_SIZE", "constexpr")]
    jobs.append(("fill_cold_global_ids_b16384", dbuf._fill_cold_global_ids_kernel, fill,
                 {"BLOCK_ROWS": 16384, "COPY_BLOCK_SIZE": 256}, 4))
    pack = ([(f"source_{c}", f32p) for c in comps] + [("source_starts", i64p),
            ("row_counts", i64p), ("output_starts", i64p), ("output", f32p),
            ("COPY_BLOCK_SIZE", "constexpr")])
    jobs.append(("pack_resident_rows", wset._pack_resident_rows_kernel, pack,
                 {"COPY_BLOCK_SIZE": 256}, 4))
    bounds = [("xyz", f32p), ("block_starts", i64p), ("block_lengths", i64p), ("output", f32p),
              ("BLOCK_ROWS", "constexpr")]
    jobs.append(("resident_block_bounds_b16384", wset._resident_block_bounds_kernel, bounds,
                 {"BLOCK_ROWS": 16384}, 8))
    return jobs


def build_triton(root: Path) -> int:
    """Compiles the jobs into TRITON_OUT/<name>/ (the .cubin, Triton's .json
    metadata and launch.json). Runs the reference modules' import under the
    CPU shims of tests/golden/reference_shim.py, so call it in a process of
    its own (the shims replace torch.cuda streams and events)."""
    import importlib.util
    import json
    import shutil
    import tempfile

    spec = importlib.util.spec_from_file_location(
        "reference_shim", HERE.parent / "tests" / "golden" / "reference_shim.py")
    shim = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(shim)
    _, dbuf, wset, gro = shim.load_reference(root)
    import triton
    from triton.backends.compiler import GPUTarget
    from triton.compiler import ASTSource

    TRITON_OUT.mkdir(parents=True, exist_ok=True)
    n = 0
    with tempfile.TemporaryDirectory() as cache:
        os.environ["TRITON_CACHE_DIR"] = cache
        for name, fn, args, constexprs, warps in _triton_jobs(dbuf, wset, gro):
            sig = dict(args)
            # every pointer 16-byte aligned and every integer a multiple of
            # 16 at the benchmark's shapes: the JIT's "D" specialization
            attrs = {(i,): [["tt.divisibility", 16]] for i, (_, t) in enumerate(args)
                     if t.startswith("*") or t == "i32"}
            src = ASTSource(fn, sig, constexprs=constexprs, attrs=attrs)
            k = triton.compile(src, target=GPUTarget("cuda", 100, 32),
                               options={"num_warps": warps})
            out = TRITON_OUT / name
            out.mkdir(exist_ok=True)
            for key, path in k.metadata_group.items():
                if key.endswith(".cubin") or key.endswith(".json"):
                    shutil.copy(path, out / key)
            (out / "launch.json").write_text(json.dumps({
                "kernel": k.name, "hash": k.hash, "args": args,
                "constexprs": {str([i for i, (a, _) in enumerate(args) if a == c][0]): v
                               for c, v in constexprs.items()},
                "constexpr_names": list(constexprs), "num_warps": warps}))
            n += 1
    return n


def load_triton_kernel(name: str):
    """(CompiledKernel, launch info) of a prebuilt reference Triton kernel,
    or None when absent. The kernel is called as kernel[grid](*args) with
    every argument in signature order, constexprs included."""
    import json
    import types

    out = TRITON_OUT / name
    info_path = out / "launch.json"
    if not info_path.exists():
        return None
    info = json.loads(info_path.read_text())
    from triton.compiler.compiler import CompiledKernel

    group = {p.name: str(p) for p in out.iterdir() if p.suffix in (".cubin", ".json")
             and p.name != "launch.json"}
    src = types.SimpleNamespace(
        signature={a: t for a, t in info["args"]},
        constants={(int(i),): v for i, v in info["constexprs"].items()},
        fn=types.SimpleNamespace(arg_names=[a for a, _ in info["args"]], launch_metadata=None))
    return CompiledKernel(src, group, info["hash"]), info


def build_if_reference_present() -> bool:
    root = reference_root()
    if root is None:
        return False
    build(root)
    if (root / "submodules" / "gsplat" / "gsplat" / "cuda" / "csrc").exists():
        build_gsplat(root)
    if (root / "strategies" / "tide_engine" / "gpu_resident_optimizer.py").exists():
        import subprocess

        subprocess.run([sys.executable, str(Path(__file__).resolve()), "--triton-only",
                        "--reference", str(root)], check=True)
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
    ap.add_argument("--triton-only", action="store_true",
                    help="only compile the reference's Triton kernels")
    args = ap.parse_args(argv)
    root = reference_root(args.reference)
    if root is None:
        print("reference tree not found; nothing built")
        return 1
    if args.triton_only:
        print("compiled", build_triton(root), "reference Triton kernels into", TRITON_OUT)
        return 0
    build(root, verbose=args.verbose)
    build_gsplat(root, verbose=args.verbose)
    print("built into", OUT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
