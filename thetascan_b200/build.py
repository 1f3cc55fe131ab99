"""Build the sm_100a shared library ``libthetascan_b200.so`` in-tree with nvcc.

The library is one translation unit (``csrc/all.cu``) exposing the C ABI of
``include/thetascan_b200.h``.  It is rebuilt when any source or the header is
newer than the library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libthetascan_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*"))) + [
        os.path.join(ROOT, "include", "thetascan_b200.h")]


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > built for s in _sources())


def nvcc_command(output: str = LIB, extra=()) -> list[str]:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
            "-Xcompiler", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
            *extra, "-o", output, os.path.join(HERE, "csrc", "all.cu")]


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    """Compile the library if it is missing or stale; return its path."""
    if force or needs_build():
        cmd = nvcc_command(extra=extra)
        if verbose:
            print(" ".join(cmd))
        tmp = LIB + ".tmp"
        cmd[cmd.index(LIB)] = tmp
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
