"""Builds the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``compute_100a``/``sm_100a`` only (B200); the
resulting ``opendipaco_b200/_C*.so`` is loaded by ``opendipaco_b200.ops``.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("opendipaco_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

NVCC = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--use_fast_math" if os.environ.get("ODP_FAST_MATH") else "-DODP_NO_FAST_MATH",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "--expt-relaxed-constexpr",
]
if os.environ.get("ODP_PTXAS_V"):
    NVCC.append("-Xptxas=-v")

setup(
    name="opendipaco_b200",
    ext_modules=[CUDAExtension("opendipaco_b200._C", sources,
                               extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
                               libraries=["cuda"])],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["opendipaco=opendipaco_b200.launch.cli:main"]},
)
