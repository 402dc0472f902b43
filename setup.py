"""Build the in-tree native extensions.

    python setup.py build_ext --inplace

* ``fak_b200._C``   -- sm_100a CUDA kernels (compiled only for compute_100a / sm_100a).
* ``fak_b200._cpu`` -- C++ runtime: CPU oracle forward, radix prefix tree, KV page allocator.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("fak_b200", "csrc")

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas", "-v" if os.environ.get("FAK_PTXAS_VERBOSE") else "-O3",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

cuda_sources = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]
cpu_sources = sorted(glob.glob(os.path.join(CSRC, "cpu", "*.cpp")))

ext_modules = [
    CUDAExtension(
        "fak_b200._C",
        cuda_sources,
        include_dirs=[os.path.join(ROOT, CSRC, "kernels")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]
if cpu_sources:
    ext_modules.append(
        CppExtension(
            "fak_b200._cpu",
            cpu_sources,
            extra_compile_args={"cxx": CXX_FLAGS + ["-march=x86-64-v3", "-pthread"]},
            extra_link_args=["-pthread"],
        )
    )

setup(
    name="fak_b200",
    version="0.1.0",
    packages=["fak_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
