"""Model shapes and modules for the parallel workloads (Llama-3-shaped)."""
from .llama import LlamaConfig, LlamaMLP, TinyLlamaStack, num_params, param_shapes  # noqa: F401
