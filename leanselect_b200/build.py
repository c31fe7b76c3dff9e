"""Build ``libleanselect_b200.so`` (sm_100a) in-tree with nvcc.

Usage: ``python -m leanselect_b200.build [--force] [--verbose]``.

The library lands in ``leanselect_b200/_lib`` next to the sources so that it
travels with a copy of the repository.  The CUDA runtime is linked
statically: the library then does not depend on which ``libcudart`` the
host process (PyTorch) loaded first.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libleanselect_b200.so"
SOURCES = ["prep.cu", "score_select.cu", "sparse_attn.cu", "capi.cu", "backbone.cu", "noalloc.cu",
           "waitprobe.cu", "select_f32.cu"]
HEADERS = ["common.cuh", "launch.h", "topk_rows.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; set NVCC or put CUDA 12.8+ on PATH")
    return cand


def _stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES + HEADERS] + sorted((ROOT / "include").glob("*.h")) + [
        Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> Path:
    """Compile every kernel for sm_100a and link the shared library."""
    if not force and not _stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    cc = nvcc()
    objects = []
    for src in SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra_flags, "-I", str(ROOT / "include"), "-c",
               str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objects, "-lpthread",
           "-ldl", "-lrt"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register/smem usage")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose, extra_flags=extra)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
