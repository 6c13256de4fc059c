"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Produces ``minispeed_b200/_C*.so``.  Every CUDA source is compiled for
Blackwell only (``-gencode arch=compute_100a,code=sm_100a``); giving an arch
flag in the nvcc arguments stops torch from adding its own arch list.
"""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("MSB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    return [os.path.relpath(p, ROOT) for p in cpp + cu]


setup(
    name="minispeed_b200",
    version="0.1.0",
    packages=find_packages(include=["minispeed_b200*"]),
    ext_modules=[
        CUDAExtension(
            name="minispeed_b200._C",
            sources=sources(),
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
