"""In-tree build of the native extensions (``python setup.py build_ext --inplace``).

* ``lightbulb_b200._C``      : sm_100a CUDA kernels (tcgen05/TMA GEMM, paged attention, ...)
* ``lightbulb_b200._native`` : host C++ (paged KV block manager, GGUF parser/dequant, CPU oracle)
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xptxas=-v" if os.environ.get("LB_PTXAS_VERBOSE") else "-Xptxas=-O3",
                     "-DNDEBUG", "-U__CUDA_NO_HALF_OPERATORS__",
                     "-U__CUDA_NO_BFLOAT16_CONVERSIONS__"]


def cuda_sources():
    return sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + \
        [os.path.join("csrc", "kernels", "bindings.cpp")]


def native_sources():
    return sorted(glob.glob(os.path.join("csrc", "native", "*.cc")))


ext = [
    CppExtension("lightbulb_b200._native", native_sources(),
                 extra_compile_args={"cxx": ["-O3", "-std=c++17"]}),
    CUDAExtension("lightbulb_b200._C", cuda_sources(),
                  include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
                  extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS}),
]

setup(name="lightbulb_b200", version="0.1.0", packages=[], ext_modules=ext,
      cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)})
