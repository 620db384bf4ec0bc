"""Tensor parallelism: process groups, collectives, fused GEMM+collective kernels."""
