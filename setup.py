"""Build for swiftllm_b200.

Two in-tree extensions:
  swiftllm_b200._core  C++17 engine core (scheduler, block manager, request
                       queue, CPU sampler, checkpoint parsers, control channel)
  swiftllm_b200._C     sm_100a CUDA kernels (tcgen05 GEMM, attention, fused
                       norms / RoPE / KV write / SwiGLU, sampling, comm)

    python setup.py build_ext --inplace            # both
    SWIFTLLM_BUILD=core python setup.py build_ext --inplace   # CPU core only

Kernels are compiled for sm_100a only:
    -gencode arch=compute_100a,code=sm_100a
"""

import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "swiftllm_b200")
WHAT = os.environ.get("SWIFTLLM_BUILD", "all")


def core_ext():
    import pybind11
    from setuptools import Extension
    srcs = sorted(glob.glob(os.path.join("swiftllm_b200", "csrc", "core", "*.cpp")))
    return Extension(
        "swiftllm_b200._core", srcs,
        include_dirs=[pybind11.get_include(), os.path.join("swiftllm_b200", "csrc", "core")],
        extra_compile_args=["-O2", "-std=c++17", "-fvisibility=hidden", "-Wno-attributes"],
        language="c++")


def cuda_ext():
    from torch.utils.cpp_extension import CUDAExtension
    srcs = sorted(glob.glob(os.path.join("swiftllm_b200", "csrc", "kernels", "*.cu"))
                  + glob.glob(os.path.join("swiftllm_b200", "csrc", "kernels", "*.cpp")))
    nvcc = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
            "-gencode", "arch=compute_100a,code=sm_100a",
            "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
            "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__"]
    if os.environ.get("SWIFTLLM_PTXAS_V") == "1":
        nvcc.append("-Xptxas=-v")
    return CUDAExtension(
        "swiftllm_b200._C", srcs,
        include_dirs=[os.path.join(PKG, "csrc", "kernels")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
    )


exts = []
cmdclass = {}
if WHAT in ("all", "core"):
    exts.append(core_ext())
if WHAT in ("all", "cuda"):
    exts.append(cuda_ext())
if exts:
    from torch.utils.cpp_extension import BuildExtension
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

setup(
    name="swiftllm_b200",
    version="0.1.0",
    packages=["swiftllm_b200", "swiftllm"],
    ext_modules=exts,
    cmdclass=cmdclass,
    entry_points={"console_scripts": ["swiftllm=swiftllm_b200.cli:main",
                                     "swiftllm-server=swiftllm_b200.server.__main__:main"]},
)
