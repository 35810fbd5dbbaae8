"""Parallelism building blocks: tensor-parallel MLP, data-parallel gradient sync."""
