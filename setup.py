"""Builds the two native extensions of axropus_deploy_b200 in place.

* ``axropus_deploy_b200._native`` -- host C++ runtime (AMF disk store, shard
  directory, controllers). Plain pybind11, no CUDA, builds on any Linux box.
* ``axropus_deploy_b200._C`` -- the sm_100a CUDA kernels and their torch bindings.
* ``axropus_deploy_b200/libkorith_b200.so`` -- the C ABI (``csrc/capi/korith.h``), a
  plain shared library that embeds the Python runtime (linked against libpython).

``python setup.py build_ext --inplace`` puts the ``.so`` files inside the package.
Set ``AXR_SKIP_CUDA=1`` to build only the host extension.
"""
import glob
import os
import subprocess
import sys
import sysconfig

import pybind11
from setuptools import Extension, setup
from setuptools.command.build_ext import build_ext as _setuptools_build_ext

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



def build_capi() -> None:
    """g++ the C ABI library next to the package (links libpython of this interpreter)."""
    site = next((p for p in sys.path if p.endswith("site-packages") and os.path.isdir(p)), "")
    libdir = sysconfig.get_config_var("LIBDIR") or "/usr/lib"
    ver = sysconfig.get_config_var("LDVERSION") or sysconfig.get_python_version()
    out = os.path.join(ROOT, "axropus_deploy_b200", "libkorith_b200.so")
    src = os.path.join(ROOT, "csrc", "capi", "korith_capi.cpp")
    if os.path.exists(out) and os.path.getmtime(out) >= max(os.path.getmtime(src), os.path.getmtime(
            os.path.join(ROOT, "csrc", "capi", "korith.h"))):
        return
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", src, "-o", out,
           "-I" + os.path.join(ROOT, "csrc", "capi"), "-I" + sysconfig.get_paths()["include"],
           f'-DAXR_SITE_PACKAGES="{site}"', "-L" + libdir, f"-lpython{ver}", "-ldl", f"-Wl,-rpath,{libdir}"]
    print(" ".join(cmd))
    subprocess.check_call(cmd)


_base_build_ext = cmdclass.get("build_ext", _setuptools_build_ext)


class build_ext_with_capi(_base_build_ext):
    def run(self):
        super().run()
        build_capi()


cmdclass["build_ext"] = build_ext_with_capi

setup(
    name="axropus_deploy_b200",
    version="0.1.0",
    packages=["axropus_deploy_b200"],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
)
