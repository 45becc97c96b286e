"""Build the sm_100a shared library ``llm_cuda_b200/_lib/libllmcuda_b200.so``.

Plain nvcc (no torch extension, no CMake): each ``csrc/*.cu`` is compiled for
``sm_100a`` only, then linked into one C-ABI shared library with the CUDA
runtime linked statically, so the library loads without a CUDA toolkit on the
library path and is found in-tree by ``llm_cuda_b200._native``.

    python -m llm_cuda_b200.build [--verbose-ptxas] [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libllmcuda_b200.so")
BUILD = os.path.join(ROOT, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "llm_cuda_b200.h"))
    objs = []
    nvcc = _nvcc()
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src] + headers):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            if not quiet:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        if not quiet:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))


if __name__ == "__main__":
    sys.exit(main())
