"""Builds libmoe_b200.so in-tree with nvcc for sm_100a.

    python -m moe_ops_b200.build [--force]

The library is one translation unit (csrc/moe_b200.cu includes every kernel header);
it is rebuilt when any file under csrc/ or include/ is newer than the .so.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
SRC = os.path.join(PKG_DIR, "csrc", "moe_b200.cu")
OUT = os.path.join(PKG_DIR, "libmoe_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2", "-shared",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _sources() -> list[str]:
    return (glob.glob(os.path.join(PKG_DIR, "csrc", "*"))
            + glob.glob(os.path.join(REPO_DIR, "include", "*.h")))


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, SRC]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
