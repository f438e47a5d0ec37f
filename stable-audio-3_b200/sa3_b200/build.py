"""Build the in-tree C-ABI library libsa3b200.so for sm_100a with nvcc.

Each `.cu` file under ``csrc/`` is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a`` and the objects are linked into
one shared library next to this file, so the library travels with the source
tree. Rebuilds only when a source or header is newer than the library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(ROOT_DIR, "csrc")
INCLUDE = os.path.join(os.path.dirname(ROOT_DIR), "include")
LIB_NAME = "libsa3b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
BUILD_DIR = os.path.join(ROOT_DIR, "_build")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsa3b200.so")
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(
        os.path.join(INCLUDE, "*.h"))


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile csrc/*.cu into libsa3b200.so (in-tree). Returns the library path."""
    if not force and not needs_build():
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-rdc=false", "-I", INCLUDE, "-c", src, "-o", obj]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if ptxas_info or verbose:
            sys.stderr.write(r.stderr)
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
