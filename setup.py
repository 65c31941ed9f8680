"""Builds the sm_100a extension in-tree: `python setup.py build_ext --inplace`.

Every CUDA source is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a); the
extension lands next to the package as ridgefill_data_b200/_C*.so.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("ridgefill_data_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    return cpp + cu


setup(
    name="ridgefill_data_b200",
    version="0.1.0",
    packages=["ridgefill_data_b200"],
    ext_modules=[
        CUDAExtension(
            name="ridgefill_data_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
