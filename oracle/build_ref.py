"""Compile the reference's own extension from its sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY (the checker and the reference arm of bench.py).

The reference (YangFan0918/flash-attention-cute) builds
``flash_attention._C`` from csrc/flash_api.cpp + csrc/flash_fwd_launch.cu
with torch's cpp_extension (setup.py:11-16).  Its CUTLASS submodule
(.gitmodules:1-3) is not vendored, so the CUTLASS/CuTe headers that ship in
this image (the copy under the flashinfer package) stand in for it.  The
reference's nvcc flags (setup.py:21-32) are kept except the architecture:
sm_86 becomes sm_100a SASS plus compute_80 PTX, so the unmodified SM80
kernel runs on a B200.  Sources are compiled where they lie; nothing of the
reference is copied into this repository.  Output: oracle/_ref/build/
flash_attention_ref_C*.so (git-ignored, shipped with the tree to GPU boxes).

    python oracle/build_ref.py [--reference-dir DIR]
"""
from __future__ import annotations

import argparse
import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref", "build")
MODULE = "flash_attention_ref_C"
DEFAULT_REFERENCE = os.environ.get("FA_REFERENCE_DIR", "/root/reference")


def cutlass_include() -> str | None:
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None
    for loc in spec.submodule_search_locations:
        cand = os.path.join(loc, "data", "cutlass", "include")
        if os.path.isdir(os.path.join(cand, "cute")):
            return cand
    return None


def built_library() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT_DIR, MODULE + "*.so")))
    return hits[0] if hits else None


def build(reference_dir: str = DEFAULT_REFERENCE, verbose: bool = False) -> str:
    srcs = [os.path.join(reference_dir, "csrc", f) for f in ("flash_api.cpp", "flash_fwd_launch.cu")]
    for s in srcs:
        if not os.path.exists(s):
            raise FileNotFoundError(f"reference source missing: {s}")
    lib = built_library()
    if lib is not None and all(os.path.getmtime(s) <= os.path.getmtime(lib) for s in srcs):
        return lib
    inc = cutlass_include()
    if inc is None:
        raise RuntimeError("no CUTLASS/CuTe headers found (flashinfer/data/cutlass/include)")
    from torch.utils.cpp_extension import load

    os.makedirs(OUT_DIR, exist_ok=True)
    load(
        name=MODULE,
        sources=srcs,
        extra_include_paths=[inc, os.path.join(reference_dir, "csrc")],
        extra_cflags=["-std=c++20", "-O3"],
        extra_cuda_cflags=[
            "-std=c++20",
            "-O3",
            "--use_fast_math",
            "--expt-relaxed-constexpr",
            "--expt-extended-lambda",
            "-gencode",
            "arch=compute_100a,code=sm_100a",
            "-gencode",
            "arch=compute_80,code=compute_80",
            "-DCUTE_SM80_ENABLED",
            "-lineinfo",
        ],
        build_directory=OUT_DIR,
        verbose=verbose,
        is_python_module=True,
    )
    lib = built_library()
    if lib is None:
        raise RuntimeError("reference build produced no library")
    return lib


def load_module():
    """Import the built reference extension (torch must be importable)."""
    import torch  # noqa: F401  (the extension links against torch)

    lib = built_library()
    if lib is None:
        raise ImportError("reference extension not built: run python oracle/build_ref.py")
    spec = importlib.util.spec_from_file_location(MODULE, lib)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=DEFAULT_REFERENCE)
    a = ap.parse_args()
    print(build(a.reference_dir, verbose=True))
    sys.exit(0)
