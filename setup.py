"""Builds the two native extensions of axropus_deploy_b200 in place.

* ``axropus_deploy_b200._native`` -- host C++ runtime (AMF disk store, shard
  directory, controllers). Plain pybind11, no CUDA, builds on any Linux box.
* ``axropus_deploy_b200._C`` -- the sm_100a CUDA kernels and their torch bindings.

``python setup.py build_ext --inplace`` puts both ``.so`` files inside the package.
Set ``AXR_SKIP_CUDA=1`` to build only the host extension.
"""
import glob
import os

import pybind11
from setuptools import Extension, setup

ROOT = os.path.dirname(os.path.abspath(__file__))
NATIVE_SRC = sorted(glob.glob(os.path.join("csrc", "native", "*.cpp")))
CXX_FLAGS = ["-O3", "-std=c++17", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]

ext_modules = [
    Extension(
        "axropus_deploy_b200._native",
        sources=NATIVE_SRC,
        include_dirs=[pybind11.get_include(), os.path.join(ROOT, "csrc", "native")],
        extra_compile_args=CXX_FLAGS,
        extra_link_args=["-lrt", "-lpthread"],
        language="c++",
    )
]
cmdclass = {}

if os.environ.get("AXR_SKIP_CUDA", "0") != "1":
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    CUDA_SRC = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + sorted(
        glob.glob(os.path.join("csrc", "kernels", "*.cpp"))
    )
    NVCC_FLAGS = [
        "-O3",
        "-std=c++17",
        "-gencode=arch=compute_100a,code=sm_100a",
        "-lineinfo",
        "--use_fast_math",
        "--expt-relaxed-constexpr",
        "-U__CUDA_NO_HALF_OPERATORS__",
        "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_OPERATORS__",
        "-Xptxas=-v" if os.environ.get("AXR_PTXAS_VERBOSE") == "1" else "-Xptxas=-O3",
    ]
    ext_modules.append(
        CUDAExtension(
            "axropus_deploy_b200._C",
            sources=CUDA_SRC,
            include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            extra_link_args=["-lcuda"],
        )
    )
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

setup(
    name="axropus_deploy_b200",
    version="0.1.0",
    packages=["axropus_deploy_b200"],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
)
