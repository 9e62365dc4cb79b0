"""Build libfa_sm100.so (the sm_100a kernels + C ABI) in-tree.

    python flash-attention-cute_b200/build_ext.py [--force]

The shared library is written next to the Python package
(``flash_attention/libfa_sm100.so``) so that it travels with the source tree;
no JIT cache and no site-packages install is involved.  The reference builds
its extension through setup.py (setup.py:7-38, sm_86 only, setup.py:28); this
build targets ``sm_100a`` only.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
PKG = os.path.join(HERE, "flash_attention")
LIB_NAME = "libfa_sm100.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

MAIN_SOURCE = os.path.join(CSRC, "fa_api.cu")
# the allocation-free split entry point (its own translation unit: it owns a
# static device scratch array and calls the public entry points above)
NOALLOC_SOURCE = os.path.join(CSRC, "fa_noalloc.cu")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")
    return cand


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "fa_sm100.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, *(extra_flags or []), f"-I{INCLUDE}", f"-I{CSRC}", "-o", tmp, MAIN_SOURCE, NOALLOC_SOURCE]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
