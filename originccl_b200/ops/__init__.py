"""Compute ops built on the library's sm_100a kernels (tensor-core GEMM, fused TP GEMM+collective)."""
from . import gemm, tp  # noqa: F401

__all__ = ["gemm", "tp"]
