"""Builds the sm_100a extension in place: python setup.py build_ext --inplace"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("trenowanie_generatora_obrazkow_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]
if os.environ.get("TGO_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="trenowanie_generatora_obrazkow_b200",
    ext_modules=[CUDAExtension(
        name="trenowanie_generatora_obrazkow_b200._C",
        sources=sources,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
