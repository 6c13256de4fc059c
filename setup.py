"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Produces ``minispeed_b200/_C*.so``.  Every CUDA source is compiled for
Blackwell only (``-gencode arch=compute_100a,code=sm_100a``); giving an arch
flag in the nvcc arguments stops torch from adding its own arch list.

``MSB_DEBUG_BUILD=1`` builds the bounds-checked variant instead,
``minispeed_b200/_C_debug*.so`` (the same sources with ``-DMSB_BOUNDS_CHECK``,
objects under their own build folder); ``MSB_DEBUG_BUILD=1`` at run time
makes the package load it.
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

DEBUG = os.environ.get("MSB_DEBUG_BUILD") == "1"
EXT_NAME = "minispeed_b200._C_debug" if DEBUG else "minispeed_b200._C"
DEFINES = ["-DMSB_BOUNDS_CHECK"] if DEBUG else []


class BuildExt(BuildExtension.with_options(use_ninja=True)):
    """The debug variant compiles into its own object folder, so the two
    builds do not overwrite each other's objects."""

    def finalize_options(self):
        super().finalize_options()
        if DEBUG:
            self.build_temp = os.path.join(self.build_temp, "bounds_check")


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
            name=EXT_NAME,
            sources=sources(),
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"] + DEFINES,
                                "nvcc": NVCC_FLAGS + DEFINES},
        )
    ],
    cmdclass={"build_ext": BuildExt},
)
