"""Build recipe for libstreamlx_cuda.so (sm_100a), in-tree.

    python -m streamlx_b200.build          # or __graft_entry__.build()

nvcc cross-compiles without a GPU.  The shared object lands next to this file
so that it travels with the repository snapshot.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libstreamlx_cuda.so")
SOURCES = ["slx_api.cu", "slx_qgemv.cu", "slx_router.cu", "slx_trunk.cu",
           "slx_pack.cu", "slx_io.cu", "slx_prefill.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False,
          extra: list[str] | None = None, out: str | None = None,
          objdir: str | None = None) -> str:
    """Compile every kernel TU and link the shared object.  ``out`` /
    ``objdir`` redirect a diagnostics build (e.g. extra=["-DSLX_TRACE"])."""
    lib_path = out or LIB
    odir = objdir or CSRC
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
            if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(ROOT, "include", "streamlx_cuda.h"))
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(odir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, *FLAGS, *(extra or []), "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(lib_path, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", lib_path, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return lib_path


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv,
          extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None)
