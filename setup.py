"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

The extension module is ``mvp_engine._C``; every kernel is compiled for
``sm_100a`` only (B200).  The arch is passed explicitly through
``extra_compile_args`` so torch's own arch list is bypassed.
"""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("mvp_engine", "ops", "csrc")

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("MVP_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")
# Debug build: device-side bounds checks on metadata-derived indices (status code 7, access skipped).
if os.environ.get("MVP_DEBUG", "0") not in ("", "0"):
    NVCC_FLAGS.append("-DMVP_DEBUG_BOUNDS")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

# torch's BuildExtension appends its own -gencode list from TORCH_CUDA_ARCH_LIST
# unless one is set; pin it to the one arch we build so no other arch sneaks in.
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

setup(
    name="mvp_engine",
    version="0.1.0",
    packages=find_packages(include=["mvp_engine*", "recipes*"]),
    ext_modules=[
        CUDAExtension(
            name="mvp_engine._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
