"""Parallelism building blocks: tensor-parallel MLP, data-parallel gradient sync, a TP x DP mesh."""
from .data_parallel import DataParallelSync, GradBuckets  # noqa: F401
from .mesh import Mesh  # noqa: F401
from .tensor_parallel import TensorParallelMLP  # noqa: F401

__all__ = ["DataParallelSync", "GradBuckets", "Mesh", "TensorParallelMLP"]
