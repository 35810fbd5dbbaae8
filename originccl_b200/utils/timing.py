"""Device timing helpers: CUDA events on the launching stream, max over ranks."""
from __future__ import annotations

from typing import Callable


def time_cuda(fn: Callable[[], None], steps: int, warmup: int, barrier: Callable[[], None] = lambda: None) -> float:
    """Runs ``warmup`` untimed calls, then times ``steps`` calls with CUDA events.

    A barrier and ``torch.cuda.synchronize()`` bracket the timed region on both sides.
    Returns milliseconds per call on this rank.
    """
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / max(steps, 1)


def max_over_ranks(value: float) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def busbw_factor(func: str, nranks: int) -> float:
    """NCCL's bus-bandwidth factors (algbw * factor = busbw)."""
    if nranks <= 1:
        return 0.0
    if func == "allreduce":
        return 2.0 * (nranks - 1) / nranks
    if func in ("allgather", "reducescatter"):
        return (nranks - 1) / nranks
    return 1.0
