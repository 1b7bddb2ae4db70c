"""Builds the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

Every kernel is compiled for ``sm_100a`` only (tcgen05 / TMA need the
architecture-specific target)."""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("atomic_ai_hybrid_b200", "csrc")
SOURCES = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

NVCC = [
    "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "--use_fast_math",
    "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("AHB_PTXAS_V") else "-DAHB_QUIET",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]

setup(
    name="atomic_ai_hybrid_b200",
    version="0.1.0",
    packages=["atomic_ai_hybrid_b200"],
    ext_modules=[
        CUDAExtension(
            name="atomic_ai_hybrid_b200._ahb_cuda",
            sources=SOURCES,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
