"""Builds the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``torchtitan_b200/_C.*.so``.  Only ``-gencode arch=compute_100a,code=sm_100a``
is emitted (B200); no other architectures are built.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("torchtitan_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("TTB_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

sources = [os.path.join(CSRC, "bindings.cpp")] + sorted(glob.glob(os.path.join(CSRC, "*.cu")))

setup(
    name="torchtitan_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="torchtitan_b200._C",
            sources=sources,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            include_dirs=[os.path.join(HERE, CSRC)],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
