"""A ``torch.distributed`` backend named ``"bccl"``: existing PyTorch code switches to this library
with ``dist.init_process_group("bccl")`` (after ``import originccl_b200.torch_backend``).

Collectives on CUDA tensors run on a device communicator for the current device (enqueued on the
current stream, like NCCL), collectives on CPU tensors on a host communicator (shared memory
between the processes of a machine, TCP between machines). Each communicator is created on the
first collective that needs it; the unique id travels through the process group's store.
Supported: all_reduce (SUM, AVG, MAX, MIN), broadcast, reduce, all_gather (list and tensor
forms), reduce_scatter (list and tensor forms), their coalesced forms (one group, i.e. one
batched kernel for small tensors), send / recv and barrier — the reference's operation set —
plus all_to_all (list form, and all_to_all_single with equal or uneven splits), gather and
scatter, which the reference does not have, as Send/Recv groups.
DistributedDataParallel runs on it unchanged; :class:`AllReduceHook` is a DDP communication hook
that fuses the gradient mean into the AllReduce and registers large bucket buffers for zero-copy.
"""
from __future__ import annotations

from typing import Dict, List

import torch
import torch.distributed as dist
from torch._C._distributed_c10d import _create_work_from_future
from torch.futures import Future

from .comm import Communicator, ReduceOp, init_from_store

_OPS = {
    dist.ReduceOp.SUM: ReduceOp.SUM,
    dist.ReduceOp.AVG: ReduceOp.AVG,
    dist.ReduceOp.MAX: ReduceOp.MAX,
    dist.ReduceOp.MIN: ReduceOp.MIN,
}


def _done(result) -> "dist.Work":
    fut: Future = Future()
    fut.set_result(result)
    return _create_work_from_future(fut)


class BcclProcessGroup(dist.ProcessGroup):
    def __init__(self, store, rank: int, world_size: int, timeout) -> None:
        super().__init__(rank, world_size)
        self._store = store
        self._timeout_ms = int(timeout.total_seconds() * 1000) if timeout is not None else 0
        self._comms: Dict[str, Communicator] = {}

    # ------------------------------------------------------------------ communicators
    def _comm(self, t: torch.Tensor) -> Communicator:
        # One device communicator per process (each rank drives its own GPU, whose index differs
        # from rank to rank), one host communicator for CPU tensors: the store key names the
        # kind only, so every rank meets under the same key.
        key = "cuda" if t.is_cuda else "cpu"
        comm = self._comms.get(key)
        if comm is None:
            device = t.device.index if t.is_cuda else -1
            comm = init_from_store(self._store, self.rank(), self.size(), key=f"bccl_pg_{key}", device=device,
                                   timeout_ms=self._timeout_ms)
            self._comms[key] = comm
        return comm

    @staticmethod
    def _op(opts) -> ReduceOp:
        if opts is None:
            return ReduceOp.SUM
        op = opts.reduceOp.op if hasattr(opts.reduceOp, "op") else opts.reduceOp
        if op not in _OPS:
            raise NotImplementedError(f"bccl: reduce op {op} is not supported (SUM, AVG, MAX, MIN are)")
        return _OPS[op]

    def getBackendName(self) -> str:
        return "bccl"

    def name(self) -> str:
        return "bccl"

    def destroy(self) -> None:
        for c in self._comms.values():
            c.destroy()
        self._comms.clear()

    # ------------------------------------------------------------------ collectives
    def allreduce(self, tensors: List[torch.Tensor], opts=None):
        op = self._op(opts)
        if len(tensors) == 1:
            self._comm(tensors[0]).all_reduce(tensors[0], op)
        else:
            self.allreduce_coalesced(tensors, opts)
        return _done(tensors)

    def allreduce_coalesced(self, tensors: List[torch.Tensor], opts=None):
        op = self._op(opts)
        comm = self._comm(tensors[0])
        with comm.group():
            for t in tensors:
                comm.all_reduce(t, op)
        return _done(tensors)

    def broadcast(self, tensors: List[torch.Tensor], opts=None):
        for t in tensors:
            self._comm(t).broadcast(t, opts.rootRank if opts is not None else 0)
        return _done(tensors)

    def reduce(self, tensors: List[torch.Tensor], opts=None):
        op = self._op(opts)
        for t in tensors:
            self._comm(t).reduce(t, opts.rootRank if opts is not None else 0, op, out=t)
        return _done(tensors)

    def _allgather_base(self, output: torch.Tensor, input: torch.Tensor, opts=None):
        self._comm(input).all_gather(output, input.contiguous())
        return _done([output])

    def allgather(self, outputs: List[List[torch.Tensor]], inputs: List[torch.Tensor], opts=None):
        for outs, inp in zip(outputs, inputs):
            flat = torch.empty(self.size() * inp.numel(), dtype=inp.dtype, device=inp.device)
            self._comm(inp).all_gather(flat, inp.contiguous())
            for r, o in enumerate(outs):
                o.copy_(flat[r * inp.numel():(r + 1) * inp.numel()].view_as(o))
        return _done(outputs)

    def allgather_into_tensor_coalesced(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor],
                                        opts=None):
        comm = self._comm(inputs[0])
        with comm.group():
            for o, i in zip(outputs, inputs):
                comm.all_gather(o, i)
        return _done(outputs)

    def _reduce_scatter_base(self, output: torch.Tensor, input: torch.Tensor, opts=None):
        self._comm(input).reduce_scatter(output, input.contiguous(), self._op(opts))
        return _done([output])

    def reduce_scatter(self, outputs: List[torch.Tensor], inputs: List[List[torch.Tensor]],
                       opts=None):
        op = self._op(opts)
        for out, ins in zip(outputs, inputs):
            flat = torch.cat([t.reshape(-1) for t in ins])
            self._comm(out).reduce_scatter(out, flat, op)
        return _done(outputs)

    def reduce_scatter_tensor_coalesced(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor],
                                        opts=None):
        op = self._op(opts)
        comm = self._comm(inputs[0])
        with comm.group():
            for o, i in zip(outputs, inputs):
                comm.reduce_scatter(o, i, op)
        return _done(outputs)

    def send(self, tensors: List[torch.Tensor], dst: int, tag: int = 0):
        for t in tensors:
            self._comm(t).send(t, dst)
        return _done(tensors)

    def recv(self, tensors: List[torch.Tensor], src: int, tag: int = 0):
        for t in tensors:
            self._comm(t).recv(t, src)
        return _done(tensors)

    def barrier(self, opts=None):
        if torch.cuda.is_available():
            torch.cuda.current_stream().synchronize()
        comm = next(iter(self._comms.values()), None)
        if comm is None:
            comm = self._comm(torch.empty(0))
        comm.barrier()
        return _done([])

    # ------------------------------------------------------------------ not in the reference
    # AllToAll, gather and scatter are not among the reference's collectives (OriginCCL
    # include/types.h:30-38); here they are Send/Recv groups (its P2P semantics: FIFO per pair,
    # one group), so they run wherever Send/Recv does.
    @staticmethod
    def _flat(t: torch.Tensor):
        """(a contiguous 1-D view of t or of a contiguous copy, the copy or None)."""
        if t.is_contiguous():
            return t.reshape(-1), None
        c = t.contiguous()
        return c.reshape(-1), c

    def alltoall_base(self, output: torch.Tensor, input: torch.Tensor, output_split_sizes: List[int],
                      input_split_sizes: List[int], opts=None):
        """dist.all_to_all_single: rows [in_off(q), in_off(q) + input_split_sizes[q]) of input (dim 0)
        go to rank q, rows from rank q land at out_off(q) of output; equal splits when the lists
        are empty (Communicator.all_to_all). One Send/Recv group."""
        comm = self._comm(input)
        w, r = comm.world_size, comm.rank
        if not output_split_sizes and not input_split_sizes:
            comm.all_to_all(output, input)
            return _done([output])
        in_rows = list(input_split_sizes) if input_split_sizes else [input.shape[0] // w] * w
        out_rows = list(output_split_sizes) if output_split_sizes else [output.shape[0] // w] * w
        if len(in_rows) != w or len(out_rows) != w or sum(in_rows) != input.shape[0] or \
                sum(out_rows) != output.shape[0] or in_rows[r] != out_rows[r]:
            raise ValueError(f"bccl: all_to_all_single split sizes {in_rows} / {out_rows} do not match "
                             f"shapes {tuple(input.shape)} / {tuple(output.shape)} on {w} ranks")
        in_row = input[0].numel() if input.shape[0] else 0
        out_row = output[0].numel() if output.shape[0] else 0
        src, _ = self._flat(input)
        dst, tmp = self._flat(output)
        io = [sum(in_rows[:q]) * in_row for q in range(w)]
        oo = [sum(out_rows[:q]) * out_row for q in range(w)]
        if out_rows[r]:
            dst[oo[r]:oo[r] + out_rows[r] * out_row].copy_(src[io[r]:io[r] + in_rows[r] * in_row])
        with comm.group():
            for q in range(w):
                if q == r:
                    continue
                if in_rows[q]:
                    comm.send(src[io[q]:io[q] + in_rows[q] * in_row], q)
                if out_rows[q]:
                    comm.recv(dst[oo[q]:oo[q] + out_rows[q] * out_row], q)
        if tmp is not None:
            output.copy_(tmp)
        return _done([output])

    def alltoall(self, outputs: List[torch.Tensor], inputs: List[torch.Tensor], opts=None):
        """dist.all_to_all: inputs[q] to rank q, outputs[q] from rank q, as one Send/Recv group."""
        comm = self._comm(inputs[0])
        r = comm.rank
        outputs[r].copy_(inputs[r])
        with comm.group():
            for q in range(comm.world_size):
                if q != r:
                    comm.send(inputs[q], q)
                    comm.recv(outputs[q], q)
        return _done(outputs)

    def gather(self, outputs: List[List[torch.Tensor]], inputs: List[torch.Tensor], opts=None):
        """dist.gather: the root receives every rank's tensor into outputs[0][q] (one group)."""
        root = opts.rootRank
        comm = self._comm(inputs[0])
        r = comm.rank
        if r != root:
            src, _ = self._flat(inputs[0])
            comm.send(src, root)
            return _done(outputs)
        outs = outputs[0]
        outs[r].copy_(inputs[0])
        tmps = []
        with comm.group():
            for q in range(comm.world_size):
                if q != r:
                    dst, tmp = self._flat(outs[q])
                    comm.recv(dst, q)
                    if tmp is not None:
                        tmps.append((outs[q], tmp))
        for o, t in tmps:
            o.copy_(t)
        return _done(outputs)

    def scatter(self, outputs: List[torch.Tensor], inputs: List[List[torch.Tensor]], opts=None):
        """dist.scatter: the root sends inputs[0][q] to rank q, which receives it into outputs[0]."""
        root = opts.rootRank
        comm = self._comm(outputs[0])
        r = comm.rank
        if r != root:
            dst, tmp = self._flat(outputs[0])
            comm.recv(dst, root)
            if tmp is not None:
                outputs[0].copy_(tmp)
            return _done(outputs)
        ins = inputs[0]
        outputs[0].copy_(ins[r])
        with comm.group():
            for q in range(comm.world_size):
                if q != r:
                    comm.send(self._flat(ins[q])[0], q)
        return _done(outputs)


class AllReduceHook:
    """DistributedDataParallel communication hook for the "bccl" backend::

        hook = AllReduceHook()
        ddp.register_comm_hook(dist.group.WORLD, hook)   # state: the bccl process group (or None)

    Each gradient bucket is averaged by ONE AllReduce with the 1/world scale fused into the
    kernel's store (DDP's default hook divides the bucket first, an extra pass over it). On CUDA,
    bucket buffers of at least ``min_bytes`` are registered with the communicator the first time
    they are seen, so their AllReduce reads and writes the peers' buffers directly (no staging).
    Every rank sees the same buckets in the same order, which keeps registration collective; DDP
    keeps its bucket buffers between iterations, so this happens once per buffer. ``close()``
    deregisters them (collective)."""

    def __init__(self, process_group: "BcclProcessGroup" = None, *, register: bool = True,
                 min_bytes: int = 1 << 20) -> None:
        self.process_group = process_group
        self.register = register
        self.min_bytes = min_bytes
        self._registered: Dict[tuple, tuple] = {}  # (ptr, bytes) -> (communicator, tensor)
        self.__name__ = self.__qualname__ = "bccl_allreduce_hook"  # DDP logs the hook's name

    def _pg(self, state) -> "BcclProcessGroup":
        for cand in (state, self.process_group, dist.distributed_c10d._get_default_group()):
            if isinstance(cand, BcclProcessGroup):
                return cand
        raise TypeError("AllReduceHook needs the 'bccl' process group")

    # No annotations: DDP compares them against the objects themselves, and this module's are
    # strings (postponed evaluation).
    def __call__(self, state, bucket):
        t = bucket.buffer()
        comm = self._pg(state)._comm(t)
        nbytes = t.numel() * t.element_size()
        if self.register and t.is_cuda and comm.world_size > 1 and nbytes >= self.min_bytes:
            key = (t.data_ptr(), nbytes)
            if key not in self._registered:
                comm.register(t)
                self._registered[key] = (comm, t)  # keeps the buffer alive while registered
        comm.all_reduce(t, ReduceOp.SUM, scale=1.0 / comm.world_size)
        fut: Future = Future()
        fut.set_result(t)
        return fut

    def close(self) -> None:
        for comm, t in self._registered.values():
            comm.deregister(t)
        self._registered.clear()


def _create(store, rank: int, world_size: int, timeout) -> BcclProcessGroup:
    return BcclProcessGroup(store, rank, world_size, timeout)


if "bccl" not in dist.Backend.backend_list:
    dist.Backend.register_backend("bccl", _create, devices=["cpu", "cuda"])
