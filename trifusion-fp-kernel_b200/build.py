"""Build the trifusion_b200 C-ABI shared library for sm_100a, in-tree.

    python trifusion-fp-kernel_b200/build.py [--force] [--jobs N]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (objects under
``_build/``) and links ``trifusion_b200/_native/libtrifusion_b200.so``.
Objects are rebuilt when their source or any header is newer. nvcc
cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
OUT_DIR = PKG_ROOT / "trifusion_b200" / "_native"
LIB = OUT_DIR / "libtrifusion_b200.so"
# Bounds-checked debug build (-DTF_DEBUG_BOUNDS): the recurrence kernel checks every
# global access against the tensors' extents, records error 2 and skips the access.
# Loaded by trifusion_b200 instead of LIB when TRIFUSION_B200_BOUNDS=1.
BOUNDS_BUILD = PKG_ROOT / "_build_bounds"
BOUNDS_LIB = OUT_DIR / "libtrifusion_b200_bounds.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-I", str(REPO / "include"), "-I", str(CSRC)]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return exe


def _headers():
    return list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))


def build(force=False, jobs=None, verbose=False, debug_bounds=False):
    """Compile and link; returns the library path (the bounds-checked one with
    ``debug_bounds``)."""
    build_dir, lib, extra = (BOUNDS_BUILD, BOUNDS_LIB, ["-DTF_DEBUG_BOUNDS"]) if debug_bounds else (BUILD, LIB, [])
    build_dir.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0)
    todo = []
    objects = []
    for src in sources:
        obj = build_dir / (src.stem + ".o")
        objects.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append((src, obj))
    exe = nvcc()

    def compile_one(item):
        src, obj = item
        cmd = [exe, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        return src.name, r.stderr

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
            for name, err in pool.map(compile_one, todo):
                if verbose and err:
                    print(f"--- {name}\n{err}", file=sys.stderr)
    if force or todo or not lib.exists():
        cmd = [exe, *ARCH, "-shared", "-o", str(lib), *map(str, objects), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill info")
    ap.add_argument("--debug-bounds", action="store_true",
                    help="build the bounds-checked library (libtrifusion_b200_bounds.so) instead")
    args = ap.parse_args()
    print(build(args.force, args.jobs, args.verbose, args.debug_bounds))


if __name__ == "__main__":
    main()
