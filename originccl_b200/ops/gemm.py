"""Tensor-core GEMM (tcgen05 + TMA + TMEM) for bf16: ``y = act(a @ w.T)``.

``w`` is stored as [N, K] (the layout of ``torch.nn.Linear.weight``), so both operands are
K-major. The kernel lives in ``csrc/kernels/gemm_sm100.cu``.
"""
from __future__ import annotations

from typing import Optional

from .. import _native

_ACTS = {None: 0, "none": 0, "silu": 1}


def available() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
    except Exception:
        return False


def gemm(a, w, activation: Optional[str] = None, out=None):
    """a: [M, K] bf16, w: [N, K] bf16 (both contiguous CUDA tensors) -> [M, N] bf16."""
    import torch
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("gemm expects bfloat16 operands")
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise ValueError(f"shape mismatch: a {tuple(a.shape)} w {tuple(w.shape)}")
    if activation not in _ACTS:
        raise ValueError(f"gemm: activation {activation!r} (none, silu)")
    if a.device != w.device or a.device.type != "cuda":
        raise ValueError(f"gemm: operands must be CUDA tensors on one device, got {a.device} and {w.device}")
    a = a.contiguous()
    w = w.contiguous()
    m, k = a.shape
    n = w.shape[0]
    if out is not None and (out.dtype != torch.bfloat16 or tuple(out.shape) != (m, n) or out.stride(1) != 1 or
                            out.device != a.device):
        raise ValueError(f"gemm: out must be a bfloat16 [{m}, {n}] tensor with unit column stride on {a.device}")
    if out is None:
        out = torch.empty(m, n, device=a.device, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    rc = _native.lib().bcclGemmBf16(a.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, out.stride(0),
                                    _ACTS[activation], stream)
    if rc != 0:
        raise RuntimeError(_native.last_error())
    return out


def kernel_name(m: int = 0, n: int = 0) -> str:
    """Which kernel an m x n GEMM uses: ``"pair_256x256"`` / ``"pair_256x224"`` (2-SM,
    cta_group::2) or ``"single_128x256"``."""
    lib = _native.lib()
    if not lib.bcclGemmUsesPair():
        return "single_128x256"
    return f"pair_256x{lib.bcclGemmTileWidth(int(m), int(n))}"


def check_error() -> int:
    """Synchronises and returns the GEMM kernels' error word (0 = no bounded wait gave up)."""
    return int(_native.lib().bcclGemmCheckError())
