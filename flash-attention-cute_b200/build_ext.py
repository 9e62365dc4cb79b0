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


# The pybind11 module (flash_attention/_fa_torch*.so): the C++ per-call path
# of forward(), linked against libfa_sm100.so through $ORIGIN.
BINDING_SOURCE = os.path.join(CSRC, "fa_torch_binding.cpp")
BINDING_NAME = "_fa_torch"


def binding_path() -> str:
    import sysconfig

    return os.path.join(PKG, BINDING_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


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


def build_binding(force: bool = False, verbose: bool = False) -> str:
    """Compile the pybind11 module with the host C++ compiler against torch's
    headers; needs libfa_sm100.so built first (it links against it)."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    out = binding_path()
    deps = [BINDING_SOURCE, os.path.join(INCLUDE, "fa_sm100.h"), os.path.abspath(__file__), LIB_PATH]
    if not force and os.path.exists(out) and all(os.path.getmtime(f) <= os.path.getmtime(out) for f in deps):
        return out
    cxx = os.environ.get("CXX") or shutil.which("g++") or "c++"
    incs = [*cpp_extension.include_paths("cuda"), sysconfig.get_paths()["include"], INCLUDE]
    libdirs = cpp_extension.library_paths("cuda")[:1]  # torch's own lib folder
    tmp = out + ".tmp"
    cmd = [
        cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
        f"-DTORCH_EXTENSION_NAME={BINDING_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
        *[f"-I{i}" for i in incs], BINDING_SOURCE, "-o", tmp,
        *[f"-L{d}" for d in libdirs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
        f"-L{PKG}", "-lfa_sm100", "-Wl,-rpath,$ORIGIN",
    ]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"binding build failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
    print(build_binding(force="--force" in sys.argv, verbose=True))
