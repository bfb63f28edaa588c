"""Build the B200 operator libraries in-tree.

* ``laplacianformer_b200/liblfb200.so`` — every CUDA kernel and the C ABI of
  ``include/laplacian_b200.h``, compiled with nvcc for sm_100a only.
* ``Laplace_subtraction_cuda*.so`` at the repository root — the PyTorch
  extension with the reference's module name and operator names
  (``setup.py``), a thin layer over liblfb200.so.

Run ``python -m laplacianformer_b200.build`` (or ``python setup.py
build_ext --inplace``, which calls :func:`build_capi` first).
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(ROOT, "_build", "capi")
LIB = os.path.join(PKG, "liblfb200.so")

CU_SOURCES = ["capi.cu", "laplace_sub.cu", "laplace_sub_packed.cu", "newton_inverse.cu", "host_pipeline.cu", "peer.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_capi(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile csrc/*.cu into liblfb200.so (incremental, parallel)."""
    os.makedirs(OBJDIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "laplacian_b200.h"))
    procs, objs = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJDIR, src.replace(".cu", ".o"))
        objs.append(o)
        if _newer(o, [s] + headers):
            cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(out.decode(errors="replace"))
            raise RuntimeError(f"nvcc failed on {src}")
    if _newer(LIB, objs):
        cmd = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


def build_extension(verbose: bool = False) -> None:
    """Build the Laplace_subtraction_cuda PyTorch extension in place."""
    build_capi(verbose=verbose)
    cmd = [sys.executable, "setup.py", "build_ext", "--inplace"]
    out = subprocess.run(cmd, cwd=ROOT, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if out.returncode != 0:
        sys.stderr.write(out.stdout.decode(errors="replace"))
        raise RuntimeError("building the Laplace_subtraction_cuda extension failed")
    if verbose:
        print(out.stdout.decode(errors="replace")[-2000:])


if __name__ == "__main__":
    build_extension(verbose="-v" in sys.argv)
