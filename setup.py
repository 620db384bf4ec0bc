"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every kernel is compiled for ``sm_100a`` only (tcgen05 / TMEM / TMA need the
arch-specific target); the module lands at ``deltaserve_vllm_b200/ops/_C*.so``.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("deltaserve_vllm_b200", "ops", "csrc")
SOURCES = [os.path.join(CSRC, f) for f in (
    "bindings.cpp", "gemm_tc.cu", "attention.cu", "norm_rope.cu", "lora_misc.cu", "peer.cu", "attn_bwd.cu",
    "tp_bwd.cu", "attn_tc.cu", "attn_bwd_tc.cu")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__",
]
if os.environ.get("DSV_PTXAS_VERBOSE") == "1":
    NVCC_FLAGS.append("-Xptxas=-v")
if os.environ.get("DSV_BOUNDS_CHECK") == "1":
    # Index checks in the paged-KV, slot and LoRA-slot reads: a bad index is
    # recorded in the device error word (ops.check_device_error) and skipped.
    NVCC_FLAGS.append("-DDSV_BOUNDS_CHECK")

setup(
    name="deltaserve_vllm_b200",
    version="0.1.0",
    packages=["deltaserve_vllm_b200"],
    ext_modules=[CUDAExtension(
        name="deltaserve_vllm_b200.ops._C",
        sources=SOURCES,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
