"""Build the in-tree sm_100a extension: ``python setup.py build_ext --inplace``."""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "bridge_b200", "csrc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
sources = [os.path.relpath(s, HERE) for s in sources]

setup(
    name="bridge_b200",
    version="0.1.0",
    packages=["bridge_b200"],
    ext_modules=[
        CUDAExtension(
            name="bridge_b200._C",
            sources=sources,
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "--use_fast_math",
                         "-Xptxas=-v" if os.environ.get("BB_PTXAS_V") else "-Xptxas=-O3"] + ARCH,
            },
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
