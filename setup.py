"""Build the avgen_b200 sm_100a CUDA extension in place.

    python setup.py build_ext --inplace

Every kernel is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`);
torch's own arch list is bypassed.
"""
from __future__ import annotations

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("avgen_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    *ARCH,
]
if os.environ.get("AVGEN_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")
if os.environ.get("AVGEN_KCHECK") == "1":  # checked build: TMA coordinates verified before each copy
    NVCC_FLAGS.append("-DAVGEN_KCHECK")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

setup(
    name="avgen_b200",
    version="0.1.0",
    packages=find_packages(include=["avgen_b200", "avgen_b200.*"]),
    package_data={"avgen_b200.simulate": ["*.json"]},
    ext_modules=[
        CUDAExtension(
            name="avgen_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["avgen=avgen_b200.cli.main:main", "avgen-b200=avgen_b200.cli.main:main"]},
)
