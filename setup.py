"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``sm_100a`` only (tcgen05 / TMA / TMEM
instructions do not exist on other architectures).
"""

import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

CSRC = os.path.join("representax_b200", "csrc")
SOURCES = [
    "bindings.cpp",
    "gemm.cu",
    "gemm_fwd.cu",
    "gemm_dgrad.cu",
    "gemm_wgrad.cu",
    "norm.cu",
    "attention.cu",
    "attention_noalloc.cu",
    "attention_tc.cu",
    "pool.cu",
    "mnr.cu",
    "optim.cu",
    "comm.cu", "pointwise.cu", "gemm_fp8.cu", "int4.cu", "mnr_tc.cu", "mxfp8.cu", "int4_gemm.cu", "attention_bwd_ws.cu", "attention_fwd_ws.cu",
]

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v",
]

setup(
    name="representax_b200",
    version="0.1.0",
    packages=find_packages(include=["representax_b200", "representax_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="representax_b200._C",
            sources=[os.path.join(CSRC, s) for s in SOURCES],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
