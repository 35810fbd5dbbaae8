"""Parallelism building blocks: tensor-parallel MLP, data-parallel gradient sync."""
from .data_parallel import DataParallelSync, GradBuckets  # noqa: F401
from .tensor_parallel import TensorParallelMLP  # noqa: F401

__all__ = ["DataParallelSync", "GradBuckets", "TensorParallelMLP"]
