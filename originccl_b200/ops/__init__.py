"""Compute ops built on the library's sm_100a kernels (tensor-core GEMM, fused TP GEMM+collective)."""
