"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``."""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("dtensor_muon_b200", "ops", "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode=arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("DMB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="dtensor_muon_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="dtensor_muon_b200._C",
            sources=sources,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
