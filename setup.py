"""Builds the b200ar native library in-tree (``python setup.py build_ext --inplace``).

Every CUDA source is compiled for sm_100a only (B200); the explicit -gencode
flag keeps torch from adding its own architecture list.

``B200AR_CHECKS=1 python setup.py build_ext --inplace`` builds the checked
debug library ``b200ar/_C_checked*.so`` instead (device-side range and epoch
checks that record errors in the status word; objects under build/checked).
Importing b200ar with ``B200AR_CHECKS=1`` in the environment loads it.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

# The image exports CC/CXX pointing at a relocated gcc wrapper; host objects that
# nvcc compiles through it throw C++ exceptions that crash during unwinding.
# The system toolchain (same gcc major version) is used instead.
for _var in ("CC", "CXX", "CUDAHOSTCXX"):
    os.environ.pop(_var, None)

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    files = []
    for pat in ("csrc/*.cpp", "csrc/**/*.cpp", "csrc/**/*.cu"):
        files += glob.glob(os.path.join(ROOT, pat), recursive=True)
    return sorted(set(os.path.relpath(f, ROOT) for f in files))


CHECKED = os.environ.get("B200AR_CHECKS") == "1"
DEFINES = ["-DB200AR_CHECKS"] if CHECKED else []

NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
] + DEFINES

setup(
    name="b200ar",
    version="0.1.0",
    packages=["b200ar"],
    ext_modules=[
        CUDAExtension(
            name="b200ar._C_checked" if CHECKED else "b200ar._C",
            sources=sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"] + DEFINES, "nvcc": NVCC_FLAGS},
            extra_link_args=["-lrt"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    options={"build": {"build_temp": os.path.join("build", "checked")}} if CHECKED else {},
)
