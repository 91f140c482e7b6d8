"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``."""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("tornado_gcm_b200", "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "--expt-extended-lambda",
    "-Xptxas=-v" if os.environ.get("TGCM_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]

setup(
    name="tornado_gcm_b200",
    version="0.1.0",
    packages=find_packages(include=["tornado_gcm_b200", "tornado_gcm_b200.*"]),
    package_data={"tornado_gcm_b200": ["configs/*.yaml", "data/*.csv", "data/*.json"]},
    ext_modules=[
        CUDAExtension(
            name="tornado_gcm_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["tornado-gcm-b200=tornado_gcm_b200.cli:main"]},
)
