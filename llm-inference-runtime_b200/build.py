"""Builds ``libpaged_attn.so`` in-tree for sm_100a with nvcc.

One translation unit (``csrc/capi.cu``) includes every kernel header, so the
library is a single nvcc invocation. The build is skipped when the library
is newer than every source.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB = os.path.join(PKG_DIR, "libpaged_attn.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def nvcc_path() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        raise RuntimeError("nvcc not found; the paged-attention library needs CUDA 12.8+")
    return nvcc


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compiles the library if needed and returns its path."""
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []), "-I" + INCLUDE, "-o", tmp,
           os.path.join(CSRC, "capi.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
