"""Build libb2attn.so in-tree with nvcc for sm_100a.

The shared library is the product's compute path: it holds every CUDA kernel
and the C ABI declared in include/b2_decode_attn.h and include/b2_block.h.  It is built next to this
file so that it travels with the source tree to the GPU host.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libb2attn.so"
SOURCES = [CSRC / "b2_attn.cu", CSRC / "b2_block.cu", CSRC / "b2_gemm.cu"]
HEADERS = [ROOT / "include" / "b2_decode_attn.h", ROOT / "include" / "b2_block.h", CSRC / "b2_internal.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def needs_build(lib: pathlib.Path = LIB) -> bool:
    if not lib.exists():
        return True
    mtime = lib.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    """Compile the CUDA sources into libb2attn.so (skipped when up to date)."""
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"),
           *map(str, SOURCES), "-o", str(tmp)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr}")
    if verbose:
        print(proc.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose=True)
    print(LIB)
