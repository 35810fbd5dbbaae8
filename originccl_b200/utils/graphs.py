"""CUDA-graph capture of collectives and of whole steps that contain them.

Every device kernel of this library finds its cross-rank sequence numbers in device memory
(advanced by the last CTA of each launch) and carries its work list in its launch parameters, so
a captured collective replays without the host: one ``cudaGraphLaunch`` runs any number of
collectives, fused TP ops and NCCL Send/Recv, and each replay synchronises with the other ranks
exactly like an eager call. Rules:

* capture with a stream-ordered communicator (the default; ``blocking=True`` communicators wait
  on the host and refuse to run while the current stream is capturing);
* every rank captures and replays the same sequence of collectives;
* run each op once eagerly before capturing it (``capture`` does): the first call of a fused
  TP op sizes its symmetric workspaces, which allocates and synchronises with the peers;
* device-side failures of replayed kernels (a bounded wait that expired, an abort) are reported
  by the next ``comm.synchronize()`` or eager call.

The reference has no device path; its closest idea is the dynamic executor's pre-planned slice
batches (OriginCCL src/executor/dynamic_multi_thread_executor.cpp:176-230).
"""
from __future__ import annotations

from typing import Callable, Optional


def capture(fn: Callable[[], object], *, repeat: int = 1, warmup: int = 3, pool=None, stream=None):
    """Runs ``fn`` ``warmup`` times eagerly on a side stream (first-use allocations, algorithm
    choice, NCCL set-up), then captures ``repeat`` back-to-back calls into one CUDA graph and
    returns it (``graph.replay()`` runs them). ``pool`` and ``stream`` are passed to
    ``torch.cuda.graph``."""
    import torch

    side = stream if stream is not None else torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, pool=pool, stream=side):
        for _ in range(repeat):
            fn()
    return g


def time_replays(graph, replays: int, calls_per_replay: int = 1, sync: Optional[Callable[[], None]] = None) -> float:
    """Device time of one captured call in microseconds: CUDA events around ``replays``
    back-to-back replays of ``graph`` on the current stream, divided by the calls they contain.
    ``sync`` (e.g. a cross-rank barrier) runs between the synchronisations before timing."""
    import torch

    torch.cuda.synchronize()
    if sync is not None:
        sync()
        torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(replays):
        graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / (replays * calls_per_replay)
