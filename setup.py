"""Build the in-tree CUDA extension ``octopus_b200._C`` for sm_100a only.

    python setup.py build_ext --inplace
"""
import glob
import os

import pybind11
from setuptools import Extension, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("octopus_b200", "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("OCTO_PTXAS_V"):
    nvcc_flags.append("-Xptxas=-v")

setup(
    name="octopus_b200",
    version="0.1.0",
    packages=["octopus_b200"],
    ext_modules=[
        Extension(
            name="octopus_b200._native",
            sources=sorted(glob.glob(os.path.join(CSRC, "native", "*.cpp"))),
            include_dirs=[pybind11.get_include()],
            extra_compile_args=["-O3", "-std=c++17", "-fvisibility=hidden"],
            language="c++",
        ),
        CUDAExtension(
            name="octopus_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},

        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
