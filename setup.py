"""Builds the in-tree CUDA extension ``nanovllm_self_b200._C`` for sm_100a only.

    python setup.py build_ext --inplace

The extension lands next to the package sources (``nanovllm_self_b200/_C*.so``) so a
copy of the repository carries it; nothing is installed into site-packages.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")
SOURCES = [
    "bindings.cpp", "gemm_bind.cpp", "comm_bind.cpp",
    "norm_act.cu", "qkv_rope_kv.cu", "attention.cu", "sampling.cu", "gemm_tcgen05.cu", "comm.cu",
    "attn_decode_noalloc.cu",
]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]

setup(
    name="nanovllm_self_b200_kernels",
    ext_modules=[
        CUDAExtension(
            name="nanovllm_self_b200._C",
            sources=[os.path.join("csrc", s) for s in SOURCES if os.path.exists(os.path.join(CSRC, s))],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
