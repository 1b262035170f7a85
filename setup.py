"""Builds the in-tree `mia_train_b200._C` extension for sm_100a (B200) only.

    python setup.py build_ext --inplace
"""

from __future__ import annotations

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("mia_train_b200", "csrc")

NVCC_FLAGS = [
    "-O3",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("MIA_PTXAS_VERBOSE") == "1":
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="mia_train_b200",
    ext_modules=[
        CUDAExtension(
            name="mia_train_b200._C",
            sources=sources,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
