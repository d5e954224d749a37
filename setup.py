"""Build the femtotron_b200 native extension in-tree for sm_100a (B200).

    python setup.py build_ext --inplace

produces femtotron_b200/_C.*.so next to the Python package.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("femtotron_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]

# FT_KERNEL_CHECKS=1: compile the in-kernel debug checks (FT_DCHECK in common.cuh)
if os.environ.get("FT_KERNEL_CHECKS") == "1":
    NVCC_FLAGS.append("-DFT_KERNEL_CHECKS")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="femtotron_b200",
    version="0.1.0",
    packages=["femtotron_b200"],
    ext_modules=[
        CUDAExtension(
            name="femtotron_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
