"""Build the in-tree native extension ``braidinfer_b200._C`` for sm_100a.

    python setup.py build_ext --inplace

nvcc cross-compiles without a GPU; the resulting .so lives inside the
package directory so it travels with the source tree.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = [os.path.join("csrc", f) for f in (
    "bindings.cpp", "gemm_tcgen05.cu", "gemm_persistent.cu", "attention.cu", "attention_tc.cu", "elementwise.cu", "sampling.cu", "comm.cu")]

NVCC = ["-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-std=c++17",
        "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        "-U__CUDA_NO_HALF_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__"]
if os.environ.get("BRAID_PTXAS_V"):
    NVCC.append("-Xptxas=-v")
CXX = ["-O3", "-std=c++17"]
# BRAID_BOUNDS_CHECK=1 builds the bounds-checked variant braidinfer_b200._C_checked
# (indices read from data are checked in the kernels; violations are recorded,
# not trapped).  Build it into its own temp directory:
#     BRAID_BOUNDS_CHECK=1 python setup.py build_ext --inplace --build-temp build/checked
CHECKED = os.environ.get("BRAID_BOUNDS_CHECK") == "1"
NAME = "braidinfer_b200._C_checked" if CHECKED else "braidinfer_b200._C"
if CHECKED:
    NVCC.append("-DBRAID_BOUNDS_CHECK")
    CXX.append("-DBRAID_BOUNDS_CHECK")

setup(
    name="braidinfer_b200",
    ext_modules=[CUDAExtension(NAME, SRC, extra_compile_args={"cxx": CXX, "nvcc": NVCC})],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
