"""Build libdcr_b200.so (the sm_100a CUDA library behind the C ABI in include/dcr_b200.h).

The library is one nvcc translation unit (csrc/dcr_b200_lib.cu) built in-tree into
``dcr_b200/lib/libdcr_b200.so`` with ``-gencode arch=compute_100a,code=sm_100a``.
It links the CUDA runtime statically and reaches the driver's tensor-map encoder through
``cudaGetDriverEntryPoint``, so it needs neither ``-lcuda`` nor a matching libcudart at
run time.

Usage: ``python -m dcr_b200.build [--force]`` (with ``dcr-attention_v3_b200`` on sys.path).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_ROOT = os.path.dirname(PKG_DIR)                 # dcr-attention_v3_b200/
REPO_ROOT = os.path.dirname(SRC_ROOT)
CSRC = os.path.join(SRC_ROOT, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libdcr_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build libdcr_b200")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(INCLUDE, "dcr_b200.h")])


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}",
           os.path.join(CSRC, "dcr_b200_lib.cu"), "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if "spill" in (r.stderr or "") and verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
