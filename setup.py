"""Builds the ``Laplace_subtraction_cuda`` PyTorch extension (the reference's
module name, setup.py:8-11 of the reference) on top of the B200 C-ABI library
laplacianformer_b200/liblfb200.so, which is compiled first with nvcc for
sm_100a.  ``python setup.py build_ext --inplace`` leaves the module at the
repository root, next to the package, so ``import Laplace_subtraction_cuda``
works from a checkout.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("lfb_build", os.path.join(HERE, "laplacianformer_b200", "build.py"))
_build = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_build)
_build.build_capi()

setup(
    name="Laplace_subtraction_cuda",
    ext_modules=[
        CUDAExtension(
            name="Laplace_subtraction_cuda",
            sources=[
                os.path.join("laplacianformer_b200", "csrc", "wrapper.cpp"),
                os.path.join("laplacianformer_b200", "csrc", "torch_ops.cpp"),
            ],
            include_dirs=[os.path.join(HERE, "include")],
            define_macros=[("WITH_CUDA", None)],
            library_dirs=[os.path.join(HERE, "laplacianformer_b200")],
            libraries=["lfb200"],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", "-Wno-unused-function"], "nvcc": []},
            extra_link_args=["-Wl,-rpath,$ORIGIN/laplacianformer_b200"],
        )
    ],
    cmdclass={"build_ext": BuildExtension},
)
