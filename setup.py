"""Build the flare_b200 native extension in-tree for sm_100a.

    python setup.py build_ext --inplace

Every CUDA source is compiled for compute_100a/sm_100a only; passing an
explicit -gencode also stops torch.utils.cpp_extension from adding its own
architecture list.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("flare_b200", "csrc")

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("FLARE_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]


def native_sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    return [os.path.relpath(s, HERE) for s in srcs]


setup(
    name="flare_b200",
    version="0.1.0",
    description="B200-native recommendation training framework",
    packages=find_packages(include=["flare_b200", "flare_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="flare_b200._C",
            sources=native_sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    python_requires=">=3.10",
)
