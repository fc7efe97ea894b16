"""Build the CUDA library of the package in place.

    python triton-mla_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (cross-compiles on a machine
without a GPU) and links them into ``triton_mla/libtriton_mla_b200.so`` with the
CUDA runtime linked statically, so the library loads on any host with an NVIDIA
driver and no CUDA toolkit.  The library needs no libcuda at link time: the one
driver entry point it uses (tensor-map encoding) is fetched at run time.  It also builds
``triton_mla/libtriton_mla_torch.so``: the decode registered as the PyTorch operator
``torch.ops.triton_mla.decode`` (g++ against the installed torch).
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
TORCH_OP_SRC = CSRC / "torch_op" / "tmla_torch_op.cpp"
TORCH_OP_LIB = PKG_ROOT / "triton_mla" / "libtriton_mla_torch.so"
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
    build_torch_op(force, verbose)
    return LIB


def build_torch_op(force: bool = False, verbose: bool = False) -> Path:
    """The PyTorch operator torch.ops.triton_mla.decode (a TORCH_LIBRARY registration over the C
    ABI), linked against the library above and against the installed torch."""
    import torch
    import torch.utils.cpp_extension as ce

    if not (force or _stale(TORCH_OP_LIB, [TORCH_OP_SRC, LIB, *INCLUDE.glob("*.h"), Path(__file__)])):
        return TORCH_OP_LIB
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in ce.include_paths("cuda")], f"-I{INCLUDE}", str(TORCH_OP_SRC), "-o", str(TORCH_OP_LIB),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           f"-L{LIB.parent}", "-ltriton_mla_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return TORCH_OP_LIB


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
