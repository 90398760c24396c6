"""Builds libtidegs_b200.so (sm_100a) in-tree with nvcc.

    python -m tidegs_b200.build            # incremental
    python -m tidegs_b200.build --force    # rebuild everything

The shared library lands in tidegs_b200/lib/ so it travels with the source
tree; object files go to _build/ at the repository root.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "tidegs_b200"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libtidegs_b200.so"

SOURCES = ("tgs_abi.cu", "tgs_adam.cu", "tgs_blocks.cu", "tgs_dirty.cu", "tgs_exchange.cu",
           "tgs_sparse.cu", "tgs_cull.cu", "tgs_render.cu", "tgs_sh.cu")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    # IEEE-rounded division and square root; no --use_fast_math, no FTZ.
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]
_IEEE_FLAGS = ("-prec-div=true", "-prec-sqrt=true", "-ftz=false")
# The render path is compared with the reference within tolerance and the
# reference builds it with fast math (gsplat setup.py:81); every other file
# keeps IEEE rounding (bit-exact parity).
FAST_MATH_SOURCES = ("tgs_render.cu", "tgs_sh.cu")


def _flags(name: str) -> list[str]:
    if name in FAST_MATH_SOURCES:
        return [f for f in NVCC_FLAGS if f not in _IEEE_FLAGS] + ["--use_fast_math"]
    return list(NVCC_FLAGS)


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the tidegs_b200 CUDA library cannot be built")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *_flags(src.name), *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c",
           str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    objs = []
    jobs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as pool:
            futs = [pool.submit(_compile, nvcc, s, o, extra, verbose or ptxas_info) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills (-Xptxas -v)")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
