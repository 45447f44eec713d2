"""Build libdsv32_int8.so in-tree with nvcc for sm_100a.

The library is one translation unit (csrc/dsv32.cu) that includes every kernel header, so the
build is a single nvcc invocation. The output lands next to this file so it travels with the
repository tree; `python -m deepseek_v32_gtx1650_b200.build` rebuilds it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libdsv32_int8.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libdsv32_int8.so")


def _sources() -> list[str]:
    out = [os.path.join(INCLUDE, "dsv32_int8.h")]
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cuh")):
            out.append(os.path.join(CSRC, f))
    return out


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/dsv32.cu into LIB_PATH (skipped when up to date). Returns the path."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = f"{LIB_PATH}.tmp{os.getpid()}"  # per process: ranks that build at once do not clobber each other
    cmd = [_nvcc(), *NVCC_FLAGS, os.path.join(CSRC, "dsv32.cu"), "-o", tmp]
    proc = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        sys.stdout.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
