"""Llama-3-shaped model pieces used by the parallel workloads.

The reference (OriginCCL) is a communication library without models; the benchmark workloads it
is measured on here are defined by their tensor shapes:

* data-parallel gradient sync for an 8B-parameter Llama-3-shaped model (``LlamaConfig.llama3_8b``
  and ``param_shapes``), and
* the tensor-parallel MLP ``SiLU(X @ W_up) @ W_down`` without a gate (``LlamaMLP``; its
  tensor-parallel form is ``originccl_b200.parallel.TensorParallelMLP``).

Weights are random-init (normal(0, 0.02)); there are no checkpoints.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch
from torch import nn


@dataclass(frozen=True)
class LlamaConfig:
    vocab_size: int = 128256
    hidden: int = 4096
    intermediate: int = 14336
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    tie_embeddings: bool = False

    @staticmethod
    def llama3_8b() -> "LlamaConfig":
        return LlamaConfig()

    @staticmethod
    def tiny() -> "LlamaConfig":
        return LlamaConfig(vocab_size=1024, hidden=256, intermediate=768, layers=2, heads=4, kv_heads=2)

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def param_shapes(cfg: LlamaConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    """(name, shape) of every parameter, in forward order (Hugging Face naming)."""
    h, f, d = cfg.hidden, cfg.intermediate, cfg.head_dim
    kv = cfg.kv_heads * d
    out: List[Tuple[str, Tuple[int, ...]]] = [("embed_tokens.weight", (cfg.vocab_size, h))]
    for i in range(cfg.layers):
        p = f"layers.{i}."
        out += [
            (p + "input_layernorm.weight", (h,)),
            (p + "self_attn.q_proj.weight", (h, h)),
            (p + "self_attn.k_proj.weight", (kv, h)),
            (p + "self_attn.v_proj.weight", (kv, h)),
            (p + "self_attn.o_proj.weight", (h, h)),
            (p + "post_attention_layernorm.weight", (h,)),
            (p + "mlp.gate_proj.weight", (f, h)),
            (p + "mlp.up_proj.weight", (f, h)),
            (p + "mlp.down_proj.weight", (h, f)),
        ]
    out.append(("norm.weight", (h,)))
    if not cfg.tie_embeddings:
        out.append(("lm_head.weight", (cfg.vocab_size, h)))
    return out


def num_params(cfg: LlamaConfig) -> int:
    total = 0
    for _, shape in param_shapes(cfg):
        n = 1
        for s in shape:
            n *= s
        total += n
    return total


class LlamaMLP(nn.Module):
    """``SiLU(x @ W_up^T) @ W_down^T`` (no gate), weights in ``nn.Linear`` layout [out, in]."""

    def __init__(self, hidden: int, ffn: int, *, dtype=torch.bfloat16, device=None, std: float = 0.02,
                 generator=None) -> None:
        super().__init__()
        self.up = nn.Parameter(torch.empty(ffn, hidden, dtype=dtype, device=device))
        self.down = nn.Parameter(torch.empty(hidden, ffn, dtype=dtype, device=device))
        with torch.no_grad():
            self.up.normal_(0.0, std, generator=generator)
            self.down.normal_(0.0, std, generator=generator)

    def forward(self, x):
        return torch.nn.functional.silu(x @ self.up.t()) @ self.down.t()


class TinyLlamaStack(nn.Module):
    """RMSNorm + MLP residual blocks with biases: a small trainable model whose gradients have both
    large matrices (bucketed by the data-parallel sync) and small vectors (synced as one group)."""

    def __init__(self, hidden: int = 256, ffn: int = 768, layers: int = 2, *, dtype=torch.float32, device=None,
                 seed: int = 0) -> None:
        super().__init__()
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.blocks = nn.ModuleList()
        for _ in range(layers):
            blk = nn.ModuleDict({
                "norm": nn.RMSNorm(hidden, dtype=dtype, device=device),
                "up": nn.Linear(hidden, ffn, bias=True, dtype=dtype, device=device),
                "down": nn.Linear(ffn, hidden, bias=True, dtype=dtype, device=device),
            })
            with torch.no_grad():
                for lin in (blk["up"], blk["down"]):
                    lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
                    lin.bias.copy_(torch.randn(lin.bias.shape, generator=g) * 0.02)
            self.blocks.append(blk)

    def forward(self, x):
        for blk in self.blocks:
            x = x + blk["down"](torch.nn.functional.silu(blk["up"](blk["norm"](x))))
        return x
