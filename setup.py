"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

The extension ``sparknet._C`` holds the symmetric-memory bootstrap (C++), the
collective kernels and the tcgen05 GEMM kernels (CUDA for sm_100a only).
"""

import os
from pathlib import Path

from setuptools import find_packages, setup

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("SPARKNET_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-Wall", "-Wno-unused-function"]


def sources():
    return sorted(str(p.relative_to(ROOT)) for p in CSRC.glob("*.c*") if p.suffix in (".cu", ".cpp"))


def ext_modules():
    from torch.utils.cpp_extension import CUDAExtension

    return [
        CUDAExtension(
            name="sparknet._C",
            sources=sources(),
            include_dirs=[str(CSRC / "include")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
            libraries=["dl"],
        )
    ]


def cmdclass():
    from torch.utils.cpp_extension import BuildExtension

    return {"build_ext": BuildExtension.with_options(use_ninja=True)}


setup(
    name="dgx-spark-networking-b200",
    version="0.1.0",
    packages=find_packages(include=["sparknet", "sparknet.*"]),
    ext_modules=ext_modules(),
    cmdclass=cmdclass(),
    package_data={"sparknet.topology": ["examples/*.json"]},
    entry_points={"console_scripts": ["sparknet=sparknet.cli:main"]},
)
