"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

The extension is compiled for Blackwell only (``-gencode arch=compute_100a,code=sm_100a``);
the flags bypass torch's own arch list.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
DEFINES = []

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas", "-v,-warn-spills",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
] + DEFINES

setup(
    name="zeroq_b200",
    version="0.1.0",
    packages=["zeroq_b200", "zeroq_b200.ops", "zeroq_b200.parallel", "zeroq_b200.models",
              "zeroq_b200.utils"],
    ext_modules=[
        CUDAExtension(
            name="zeroq_b200._C",
            sources=SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"] + DEFINES, "nvcc": NVCC_FLAGS},
            libraries=["cublas"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
