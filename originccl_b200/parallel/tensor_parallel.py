"""Tensor-parallel (sequence-parallel) MLP: ``out = reduce_scatter(silu(all_gather(x) @ W_up.T) @ W_down.T)``.

Activations enter and leave sequence-sharded ([tokens/world, hidden] per rank); W_up is split by
rows (columns of the up projection), W_down by columns, as in Megatron-LM. The forward pass is two
fused kernels (:mod:`originccl_b200.ops.tp`); :meth:`forward_reference` runs the same math with
NCCL collectives and cuBLAS GEMMs for comparison.
"""
from __future__ import annotations


class TensorParallelMLP:
    def __init__(self, comm, hidden: int, ffn: int, *, seed: int = 0, std: float = 0.02, device=None) -> None:
        import torch
        world = comm.world_size
        if ffn % world != 0:
            raise ValueError("ffn must divide evenly over the ranks")
        self.comm = comm
        self.hidden, self.ffn, self.world = hidden, ffn, world
        self.ffn_shard = ffn // world
        dev = device if device is not None else torch.device("cuda", max(comm.device, 0))
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + comm.rank)
        # nn.Linear layout: up [ffn_shard, hidden], down [hidden, ffn_shard]
        self.w_up = (torch.randn(self.ffn_shard, hidden, device=dev, generator=g) * std).bfloat16()
        self.w_down = (torch.randn(hidden, self.ffn_shard, device=dev, generator=g) * std).bfloat16()

    def forward(self, x_shard, stream=None):
        from ..ops import tp
        h = tp.all_gather_gemm(self.comm, x_shard, self.w_up, "silu", stream=stream)
        return tp.gemm_reduce_scatter(self.comm, h, self.w_down, stream=stream)

    __call__ = forward

    def forward_reference(self, x_shard, group=None):
        """Same math through torch.distributed (NCCL) and cuBLAS."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return torch.nn.functional.silu(x_shard @ self.w_up.t()) @ self.w_down.t()
        x = torch.empty(x_shard.shape[0] * self.world, self.hidden, device=x_shard.device, dtype=x_shard.dtype)
        dist.all_gather_into_tensor(x, x_shard, group=group)
        h = torch.nn.functional.silu(x @ self.w_up.t())
        partial = h @ self.w_down.t()
        out = torch.empty(x_shard.shape[0], self.hidden, device=x_shard.device, dtype=x_shard.dtype)
        dist.reduce_scatter_tensor(out, partial, group=group)
        return out
