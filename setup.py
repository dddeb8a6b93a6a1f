"""Build the sm_100a CUDA extension of ditserve_b200 in-tree.

    python setup.py build_ext --inplace

Every .cu file is compiled for compute_100a/sm_100a only (B200).  Passing
-gencode explicitly makes torch skip its own architecture list.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("ditserve_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("DS_PTXAS_VERBOSE") else "-O3",
]

ext = CUDAExtension(
    name="ditserve_b200._C",
    sources=[
        os.path.join(CSRC, "bindings.cpp"),
        os.path.join(CSRC, "gemm.cu"),
        os.path.join(CSRC, "attention.cu"),
        os.path.join(CSRC, "elementwise.cu"),
        os.path.join(CSRC, "comm.cu"),
        os.path.join(CSRC, "noalloc.cu"),
        os.path.join(CSRC, "ring_codec.cu"),
        os.path.join(CSRC, "conv.cu"),
    ],
    include_dirs=[os.path.join(HERE, CSRC)],
    extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
)

setup(
    name="ditserve_b200",
    version="0.1.0",
    packages=["ditserve_b200"],
    ext_modules=[ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
