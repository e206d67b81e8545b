"""Builds libb2g.so (the C-ABI GEMM / pack library) in-tree for sm_100a.

    python -m gfx950_gluon_tutorials_b200.build [--force]

nvcc cross-compiles without a GPU; the shared object lands next to this file
so it travels with the repository to the GPU host.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_PATH = os.path.join(PKG_DIR, "libb2g.so")

SOURCES = ["capi.cu", "pack.cu", "noalloc.cu", "attention.cu"]
HEADERS = ["ptx.cuh", "sched.h", "gemm_kernel.cuh", "skinny_kernel.cuh", "pack.cuh",
           "capi_internal.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE, "b2g.h"))
    return files


def needs_build(lib: str = LIB_PATH) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if a source is newer than it; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        f"-I{INCLUDE}",
        "-DB2G_EXPORT",
        *[os.path.join(CSRC, s) for s in SOURCES],
        "-o",
        tmp,
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
