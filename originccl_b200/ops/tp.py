"""Fused tensor-parallel GEMM + collective ops (sequence-parallel Megatron-style MLP blocks).

* :func:`all_gather_gemm` -- ``y = act(all_gather(x_shard) @ w.T)``: one kernel pushes this rank's
  token shard into every peer's gathered buffer over NVLink while the tcgen05 GEMM consumes the
  row blocks that have arrived.
* :func:`gemm_reduce_scatter` -- ``out = reduce_scatter(h @ w.T)`` over tokens: one kernel writes
  every partial output tile straight into its owner's staging buffer as the GEMM produces it,
  and the owner sums the partials as they complete.

Weights use the ``nn.Linear`` layout ([out_features, in_features]). Shards must have a multiple
of 128 rows. Both ops are collective: every rank of the communicator calls them together.
"""
from __future__ import annotations

from typing import Optional

from .. import _native

_ACTS = {None: 0, "none": 0, "silu": 1}


def _stream(comm, stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream(comm.device)
    return int(stream.cuda_stream if hasattr(stream, "cuda_stream") else stream), 1


def all_gather_gemm(comm, x_shard, w, activation: Optional[str] = None, out=None, stream=None):
    """x_shard [ms, k] bf16, w [n, k] bf16 -> [world*ms, n] bf16."""
    import torch
    ms, k = x_shard.shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(ms * comm.world_size, n, device=x_shard.device, dtype=torch.bfloat16)
    s, has = _stream(comm, stream)
    rc = _native.lib().bcclTpAllGatherGemm(comm._h, x_shard.data_ptr(), w.data_ptr(), out.data_ptr(), ms, k, n,
                                           _ACTS[activation], s, has)
    if rc != 0:
        raise RuntimeError(_native.last_error())
    return out


def gemm_reduce_scatter(comm, h, w, out=None, stream=None):
    """h [world*ms, k] bf16, w [n, k] bf16 -> this rank's rows [ms, n] of sum_ranks(h @ w.T)."""
    import torch
    m, k = h.shape
    n = w.shape[0]
    ms = m // comm.world_size
    if out is None:
        out = torch.empty(ms, n, device=h.device, dtype=torch.bfloat16)
    s, has = _stream(comm, stream)
    rc = _native.lib().bcclTpGemmReduceScatter(comm._h, h.data_ptr(), w.data_ptr(), out.data_ptr(), ms, k, n, s, has)
    if rc != 0:
        raise RuntimeError(_native.last_error())
    return out
