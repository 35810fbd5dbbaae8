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


def _check(name, a, w, out, out_shape, activation=None):
    """Operands of a fused op: 2-D bf16 CUDA tensors on one device, a's columns = w's columns,
    out (if given) contiguous bf16 of out_shape. Returns a and w made contiguous (the kernels
    read row-major operands through TMA)."""
    import torch
    if activation not in _ACTS:
        raise ValueError(f"{name}: activation {activation!r} (none, silu)")
    for what, t in (("input", a), ("weight", w)) + ((("out", out),) if out is not None else ()):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: {what} must be bfloat16, got {t.dtype}")
        if t.dim() != 2:
            raise ValueError(f"{name}: {what} must be 2-D, got shape {tuple(t.shape)}")
    if a.shape[1] != w.shape[1]:
        raise ValueError(f"{name}: input {tuple(a.shape)} and weight {tuple(w.shape)} differ in K")
    if out is not None and (tuple(out.shape) != tuple(out_shape) or not out.is_contiguous()):
        raise ValueError(f"{name}: out must be a contiguous {tuple(out_shape)} tensor, got {tuple(out.shape)}")
    devs = {t.device for t in (a, w) + ((out,) if out is not None else ())}
    if len(devs) != 1 or next(iter(devs)).type != "cuda":
        raise ValueError(f"{name}: operands must be CUDA tensors on one device, got {sorted(map(str, devs))}")
    return a.contiguous(), w.contiguous()


def all_gather_gemm(comm, x_shard, w, activation: Optional[str] = None, out=None, stream=None):
    """x_shard [ms, k] bf16, w [n, k] bf16 -> [world*ms, n] bf16."""
    import torch
    ms, n = x_shard.shape[0], w.shape[0]
    x_shard, w = _check("all_gather_gemm", x_shard, w, out, (ms * comm.world_size, n), activation)
    k = x_shard.shape[1]
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
    m, n = h.shape[0], w.shape[0]
    if m % comm.world_size:
        raise ValueError(f"gemm_reduce_scatter: {m} rows do not split over {comm.world_size} ranks")
    ms = m // comm.world_size
    h, w = _check("gemm_reduce_scatter", h, w, out, (ms, n))
    k = h.shape[1]
    if out is None:
        out = torch.empty(ms, n, device=h.device, dtype=torch.bfloat16)
    s, has = _stream(comm, stream)
    rc = _native.lib().bcclTpGemmReduceScatter(comm._h, h.data_ptr(), w.data_ptr(), out.data_ptr(), ms, k, n, s, has)
    if rc != 0:
        raise RuntimeError(_native.last_error())
    return out
