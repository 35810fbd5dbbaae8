"""Data-parallel gradient-sync cases, run inside each rank process (host-memory communicator)."""
from __future__ import annotations

from typing import Dict


def _grads_for(rank: int, model_seed: int, hidden: int):
    """Gradients of a TinyLlamaStack on rank ``rank``'s batch (computed locally, no communication)."""
    import torch
    from originccl_b200.models import TinyLlamaStack
    m = TinyLlamaStack(hidden=hidden, ffn=3 * hidden, layers=2, seed=model_seed)
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(16, hidden, generator=g)
    m(x).pow(2).mean().backward()
    return {n: p.grad.clone() for n, p in m.named_parameters()}


def run_dp_sync(rank: int, world: int, mode: str, bucket_bytes: int) -> Dict:
    import torch
    from originccl_b200 import init_from_env
    from originccl_b200.models import TinyLlamaStack
    from originccl_b200.parallel.data_parallel import DataParallelSync, GradBuckets

    hidden = 64
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    model = TinyLlamaStack(hidden=hidden, ffn=3 * hidden, layers=2, seed=7)
    grads = GradBuckets(model.named_parameters(), bucket_bytes=bucket_bytes, small_bytes=1024)
    dp = DataParallelSync(comm, grads, register=True)  # registration: a no-op for host memory
    if mode == "attach":
        dp.attach()
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(16, hidden, generator=g)
    for step in range(2):  # the second step checks that the hooks re-arm and accumulation restarts
        grads.zero_()
        model(x).pow(2).mean().backward()
        if mode == "attach":
            dp.finish()
        else:
            dp.sync()
    expect = [_grads_for(r, 7, hidden) for r in range(world)]
    worst = 0.0
    for n, p in model.named_parameters():
        ref = sum(e[n] for e in expect) / world
        worst = max(worst, (p.grad - ref).abs().max().item())
        assert torch.allclose(p.grad, ref, rtol=1e-5, atol=1e-6), f"{n}: max diff {(p.grad - ref).abs().max()}"
    out = {"buckets": grads.num_buckets, "small": len(grads.small_idx), "worst": worst}
    dp.close()
    comm.destroy()
    return out
