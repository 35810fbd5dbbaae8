"""Data-parallel gradient synchronisation: bucketed AllReduce with a fused 1/world scale.

Gradients live in one flat buffer per dtype, laid out in reverse parameter order (the order in
which backward produces them), and are synced in fixed-size buckets (25 MiB by default) that are
plain slices of that buffer, so a bucket needs no packing copy. Each bucket is one
``all_reduce(SUM, scale=1/world)``: the mean is fused into the collective's store instead of a
separate ``div_`` pass over 16 GB. Tensors no larger than ``small_bytes`` (biases, norm weights)
are kept out of the buckets and synced as ONE ``GroupStart``/``GroupEnd`` batch, which the
library turns into a single batched kernel.

Parity: the reference has no training code; its AVG reduction (OriginCCL src/utils.cpp:372-410)
and GroupStart/GroupEnd batching (src/communicator.cpp:350-401) are the primitives this builds on.

Two ways to use it::

    grads = GradBuckets(model.named_parameters(), device="cuda")   # gradients become bucket views
    dp = DataParallelSync(comm, grads)
    loss.backward(); dp.sync()                                      # after backward

    dp.attach()                     # or overlap with backward: buckets launch as they fill
    loss.backward(); dp.finish()

On GPUs with more than one rank the bucket storage is registered with the communicator by default
(``register=None``): the peers address it, so each bucket is reduced over NVLink peer memory in
one kernel without staging copies (on 4 x B200, a Llama-3-8B-shaped gradient sync ran 1.31x
NCCL's time registered and 0.88x staged). ``register=False`` keeps the staged path; call
:meth:`DataParallelSync.close` before the gradients are freed.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple, Union

import torch

from ..comm import BcclError, ReduceOp

ShapeSpec = Tuple[str, Tuple[int, ...]]


class GradBuckets:
    """Flat gradient storage for a set of parameters (or bare shapes) split into buckets.

    ``params`` is an iterable of ``(name, nn.Parameter)`` or ``(name, shape)``. For parameters,
    ``.grad`` is set to a view into the flat storage, so autograd accumulates in place.
    ``allocator(shape, dtype)`` provides the bucketed storage instead of ``torch.zeros``; with
    ``comm.symmetric_empty`` the buckets live in multicast-bound memory and, where the planner
    picks NVLS, are reduced in place without staging copies.
    """

    def __init__(self, params: Iterable[Tuple[str, Union[torch.nn.Parameter, Sequence[int]]]], *,
                 dtype: Optional[torch.dtype] = None, device=None, bucket_bytes: int = 25 << 20,
                 small_bytes: int = 4096, allocator=None) -> None:
        items = list(params)
        if not items:
            raise ValueError("no parameters")
        self.params: List[Optional[torch.nn.Parameter]] = []
        self.names: List[str] = []
        shapes: List[Tuple[int, ...]] = []
        for name, p in items:
            self.names.append(name)
            if isinstance(p, torch.Tensor):
                self.params.append(p)
                shapes.append(tuple(p.shape))
                dtype = dtype or p.dtype
                device = device if device is not None else p.device
            else:
                self.params.append(None)
                shapes.append(tuple(int(s) for s in p))
        self.dtype = dtype or torch.bfloat16
        self.device = torch.device(device if device is not None else "cpu")
        es = torch.empty((), dtype=self.dtype).element_size()
        if bucket_bytes < es:
            raise ValueError("bucket_bytes too small")
        numels = [_numel(s) for s in shapes]
        self.small_idx = [i for i, n in enumerate(numels) if n * es <= small_bytes]
        large = [i for i, n in enumerate(numels) if n * es > small_bytes]
        large.reverse()  # backward produces the last parameters' gradients first
        n_large = sum(numels[i] for i in large)
        if allocator is not None:  # e.g. comm.symmetric_empty: buckets the collectives read in place
            self.flat = allocator((n_large,), self.dtype).zero_()
        else:
            self.flat = torch.zeros(n_large, dtype=self.dtype, device=self.device)
        self.small_flat = torch.zeros(sum(numels[i] for i in self.small_idx), dtype=self.dtype, device=self.device)
        self.views: List[torch.Tensor] = [torch.empty(0)] * len(items)
        self.offsets: List[int] = [0] * len(items)
        off = 0
        for i in large:
            self.views[i] = self.flat[off:off + numels[i]].view(shapes[i])
            self.offsets[i] = off
            off += numels[i]
        soff = 0
        for i in self.small_idx:
            self.views[i] = self.small_flat[soff:soff + numels[i]].view(shapes[i])
            soff += numels[i]
        self.large_idx = large
        self.bucket_numel = max(1, bucket_bytes // es)
        total = self.flat.numel()
        self.bucket_bounds = [(b, min(b + self.bucket_numel, total)) for b in range(0, total, self.bucket_numel)]
        for p, v in zip(self.params, self.views):
            if p is not None:
                p.grad = v

    @property
    def num_buckets(self) -> int:
        return len(self.bucket_bounds)

    def bucket(self, i: int) -> torch.Tensor:
        lo, hi = self.bucket_bounds[i]
        return self.flat[lo:hi]

    def small_tensors(self) -> List[torch.Tensor]:
        return [self.views[i] for i in self.small_idx]

    def buckets_of(self, i: int) -> range:
        """Indices of the buckets that parameter ``i`` (a large one) overlaps."""
        lo = self.offsets[i]
        hi = lo + self.views[i].numel()
        return range(lo // self.bucket_numel, (hi - 1) // self.bucket_numel + 1)

    def zero_(self) -> None:
        self.flat.zero_()
        self.small_flat.zero_()

    @property
    def numel(self) -> int:
        return self.flat.numel() + self.small_flat.numel()


def _numel(shape: Sequence[int]) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


class DataParallelSync:
    """Averages :class:`GradBuckets` over the ranks of ``comm`` (a :class:`~originccl_b200.Communicator`).

    All ranks must sync the same buckets in the same order; both :meth:`sync` and the hooks of
    :meth:`attach` launch buckets strictly in index order. The hooks run on the autograd thread
    and call the communicator from there: do not use the same communicator from another thread
    while backward runs.
    """

    def __init__(self, comm, grads: GradBuckets, *, average: bool = True, stream=None,
                 register: Optional[bool] = None) -> None:
        self.comm = comm
        self.grads = grads
        # Registered: the peers map the bucket storage (CUDA IPC), so every bucket is reduced in
        # place over peer memory without staging copies (collective; call close() before the
        # gradients are freed). None: register where possible, else stay staged; memory from
        # cuMemCreate (symmetric allocations, expandable segments) has no IPC handle, and every
        # rank learns that in the same collective, so all of them fall back together.
        want = (register is None or bool(register)) and grads.device.type == "cuda" and comm.world_size > 1
        self.registered = False
        if want:
            try:
                comm.register(grads.flat)
                self.registered = True
            except BcclError:
                if register:
                    raise
        self.scale = 1.0 / comm.world_size if average else 1.0
        self.on_gpu = grads.device.type == "cuda"
        if self.on_gpu and stream is None:
            stream = torch.cuda.Stream(device=grads.device)
        self.stream = stream
        self._bucket_batch = comm.batch([grads.bucket(i) for i in range(grads.num_buckets)])
        self._small_batch = comm.batch(grads.small_tensors())
        self._hooks: list = []
        self._pending: List[int] = []
        self._next = 0

    def close(self) -> None:
        """Collective when registered: releases the peers' mappings of the bucket storage."""
        self.detach()
        if self.registered:
            self.comm.deregister(self.grads.flat)
            self.registered = False

    # ------------------------------------------------------------------ after-backward sync
    def sync(self, stream=None) -> None:
        """Launches every bucket, then the small tensors as one group, on ``stream`` (default: the
        current stream, so later work on it sees averaged gradients)."""
        s = stream if stream is not None else (torch.cuda.current_stream(self.grads.device) if self.on_gpu else None)
        # One library call for all buckets (each its own AllReduce, in order) and one for the
        # small tensors (one group, i.e. one batched kernel).
        self.comm.all_reduce_many(self._bucket_batch, ReduceOp.SUM, scale=self.scale, grouped=False, stream=s)
        self._sync_small(s)

    def _sync_small(self, s) -> None:
        if self._small_batch.n:
            self.comm.all_reduce_many(self._small_batch, ReduceOp.SUM, scale=self.scale, grouped=True, stream=s)

    # ------------------------------------------------------------------ overlap with backward
    def attach(self) -> None:
        """Registers hooks so that each bucket's AllReduce starts (on this object's stream) as soon
        as every gradient it holds has been accumulated. Call :meth:`finish` after backward."""
        if self._hooks:
            return
        for i in self.grads.large_idx:
            p = self.grads.params[i]
            if p is None:
                raise ValueError("attach() needs parameters, not bare shapes")
            self._hooks.append(p.register_post_accumulate_grad_hook(self._make_hook(i)))
        self._reset()

    def detach(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()

    def _reset(self) -> None:
        self._pending = [0] * self.grads.num_buckets
        for i in self.grads.large_idx:
            for b in self.grads.buckets_of(i):
                self._pending[b] += 1
        self._next = 0

    def _make_hook(self, i: int):
        def hook(_p) -> None:
            for b in self.grads.buckets_of(i):
                self._pending[b] -= 1
            self._launch_ready()
        return hook

    def _launch_ready(self) -> None:
        while self._next < self.grads.num_buckets and self._pending[self._next] == 0:
            b = self._next
            if self.on_gpu:
                self.stream.wait_stream(torch.cuda.current_stream(self.grads.device))
            self.comm.all_reduce(self.grads.bucket(b), ReduceOp.SUM, scale=self.scale,
                                 stream=self.stream if self.on_gpu else None)
            self._next += 1

    def finish(self) -> None:
        """Launches what the hooks have not (buckets and the small group), then makes the current
        stream wait for all of it. Every large gradient must have been produced by then."""
        if any(self._pending[b] for b in range(self._next, self.grads.num_buckets)):
            raise RuntimeError("finish() before every bucketed gradient was accumulated")
        if self.on_gpu:
            self.stream.wait_stream(torch.cuda.current_stream(self.grads.device))
        self._sync_small(self.stream if self.on_gpu else None)
        if self.on_gpu:
            torch.cuda.current_stream(self.grads.device).wait_stream(self.stream)
        self._reset()
