"""Ahead-of-time build of the native extension for sm_100a (B200).

    python setup.py build_ext --inplace

builds ``quantized_flash_communication_b200/_C*.so`` in the source tree.  Every CUDA
source is compiled with ``-gencode arch=compute_100a,code=sm_100a`` only; torch's own
arch list is bypassed.  No GPU is needed to build (nvcc cross-compiles).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = "quantized_flash_communication_b200"
CSRC = os.path.join(PKG, "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("QFC_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
cxx_flags = ["-O3", "-std=c++17", "-ffp-contract=off", "-DNDEBUG"]

setup(
    name=PKG,
    version="0.1.0",
    packages=[PKG],
    ext_modules=[
        CUDAExtension(
            name=f"{PKG}._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": cxx_flags, "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
