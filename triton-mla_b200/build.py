"""Build the CUDA library of the package in place.

    python triton-mla_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (cross-compiles on a machine
without a GPU) and links them into ``triton_mla/libtriton_mla_b200.so`` with the
CUDA runtime linked statically, so the library loads on any host with an NVIDIA
driver and no CUDA toolkit.  The library needs no libcuda at link time: the one
driver entry point it uses (tensor-map encoding) is fetched at run time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB = PKG_ROOT / "triton_mla" / "libtriton_mla_b200.so"
OBJ_DIR = PKG_ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-Wall", "-diag-suppress", "177"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> Path:
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    objs = []
    for src in sources():
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra_flags, "-I", str(INCLUDE), "-I", str(CSRC),
                   "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    lib = build(force=args.force or args.ptxas_info, verbose=args.verbose, extra_flags=extra)
    print(f"built {lib}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
