"""Builds the in-tree CUDA library ``opengenie_b200/libogx.so`` for sm_100a with nvcc.

The library is one translation unit (csrc/ogx_capi.cu) so the device status word
and the kernels share one module.  It links the CUDA runtime statically and reaches
the driver's tensor-map encoder through cudaGetDriverEntryPoint, so loading it needs
no libcuda on a machine without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
SOURCES = [os.path.join(CSRC, "ogx_capi.cu")]
DEPENDS = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
    os.path.join(os.path.dirname(PKG_DIR), "include", "ogx.h")
]
OUTPUT = os.path.join(PKG_DIR, "libogx.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def up_to_date() -> bool:
    if not os.path.exists(OUTPUT):
        return False
    out_m = os.path.getmtime(OUTPUT)
    return all(os.path.getmtime(p) <= out_m for p in DEPENDS if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles libogx.so unless it is newer than every source; returns its path."""
    if not force and up_to_date():
        return OUTPUT
    cmd = [nvcc(), *NVCC_FLAGS, "-o", OUTPUT + ".tmp", *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(OUTPUT + ".tmp", OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
