"""Compile the reference operators from their own sources into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The reference (BirdWithDreams/LaplacianFormer) is a
PyTorch CUDA extension whose sources are five files (src/wrapper.cpp,
src/LaplaceSubtraction_cuda.cu, src/LaplaceSubtraction_cuda_kernel.cu,
src/NewtonInverse_cuda_kernel.cu, src/cuda_version.cu) plus include/.  This
recipe compiles them where they lie — it does not run the reference's
setup.py — with the reference's own compiler flags (setup.py:22-33: WITH_CUDA,
-O3, --use_fast_math, --expt-relaxed-constexpr, -lineinfo) for sm_100, under
the module name ``Laplace_subtraction_cuda_ref`` so it can be imported next to
the B200 module.  Output: oracle/_ref/Laplace_subtraction_cuda_ref.so (not
committed; it travels to the GPU box with the working tree).

Usage: python oracle/build_ref.py [REFERENCE_ROOT]

REFERENCE_ROOT is the reference checkout: the argument, else the
LF_REFERENCE_ROOT environment variable, else a ``reference`` directory next
to this repository.
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "Laplace_subtraction_cuda_ref"


def default_root() -> str:
    """The reference checkout: $LF_REFERENCE_ROOT, else ../reference beside the repository."""
    env = os.environ.get("LF_REFERENCE_ROOT")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build(ref_root: str | None = None, verbose: bool = False) -> str:
    from torch.utils.cpp_extension import load

    ref_root = ref_root or default_root()
    src = os.path.join(ref_root, "src")
    sources = [
        os.path.join(src, f)
        for f in ("wrapper.cpp", "LaplaceSubtraction_cuda.cu", "LaplaceSubtraction_cuda_kernel.cu",
                  "NewtonInverse_cuda_kernel.cu", "cuda_version.cu")
    ]
    for s in sources:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    load(
        name=NAME,
        sources=sources,
        extra_include_paths=[os.path.join(ref_root, "include")],
        extra_cflags=["-O3", "-std=c++17", "-Wno-unused-function", "-DWITH_CUDA"],
        extra_cuda_cflags=["-O3", "-std=c++17", "--expt-relaxed-constexpr", "--use_fast_math", "-lineinfo",
                           "-DWITH_CUDA", "-gencode=arch=compute_100,code=sm_100"],
        build_directory=OUT,
        verbose=verbose,
        is_python_module=True,
    )
    return os.path.join(OUT, NAME + ".so")


def load_ref():
    """Import the prebuilt reference module from oracle/_ref (None if absent)."""
    path = os.path.join(OUT, NAME + ".so")
    if not os.path.exists(path):
        return None
    import importlib.util

    import torch  # noqa: F401  (the module links against torch)

    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
