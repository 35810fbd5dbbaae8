"""Python front end of the communicator.

Mirrors the reference's API (OriginCCL include/communicator.h:19-75) in Python naming:
``get_unique_id``, ``init``, ``finalize``, ``all_reduce``, ``broadcast``, ``reduce``,
``all_gather``, ``reduce_scatter``, ``send``, ``recv``, ``group_start``/``group_end`` (or the
``group()`` context manager), and the local/machine views. Buffers are torch tensors (CPU for a
host communicator, CUDA for a device communicator) or, for host communicators, numpy arrays.

Device communicators enqueue on the caller's current torch CUDA stream by default and return
immediately (like ``torch.distributed``); pass ``blocking=True`` to run on the library's own
stream and wait for the result (the reference's synchronous contract).
"""
from __future__ import annotations

import contextlib
import ctypes
import enum
import os
import time
from dataclasses import dataclass
from typing import Any, Optional, Sequence

from . import _native


class DataType(enum.IntEnum):
    FLOAT32 = 0
    FLOAT64 = 1
    INT32 = 2
    INT64 = 3
    BF16 = 4
    FP16 = 5


class ReduceOp(enum.IntEnum):
    SUM = 0
    MAX = 1
    MIN = 2
    AVG = 3


class Algo(enum.IntEnum):
    AUTO = 0
    ONESHOT = 1
    TWOSHOT = 2
    NVLS = 3
    RING = 4
    HYBRID = 5  # AllReduce: part through the switch (NVLS), the rest two-shot, in one launch
    LL = 6      # AllReduce / AllGather / ReduceScatter up to 2 MiB per rank: data and epoch flags in one store, no barrier


class CollFunc(enum.IntEnum):
    ALLREDUCE = 0
    BROADCAST = 1
    REDUCE = 2
    ALLGATHER = 3
    REDUCESCATTER = 4
    SEND = 5
    RECV = 6


_DTYPE_SIZE = {DataType.FLOAT32: 4, DataType.FLOAT64: 8, DataType.INT32: 4, DataType.INT64: 8,
               DataType.BF16: 2, DataType.FP16: 2}


class BcclError(RuntimeError):
    """A library call returned failure; the message is the library's last error."""


@dataclass(frozen=True)
class UniqueId:
    ip_addr: str
    port: int

    def to_bytes(self) -> bytes:
        return f"{self.ip_addr}:{self.port}".encode()

    @staticmethod
    def from_bytes(b: bytes) -> "UniqueId":
        ip, port = b.decode().rsplit(":", 1)
        return UniqueId(ip, int(port))


_DTYPE_CACHE: dict = {}  # torch / numpy dtype object -> DataType


def _resolve_dtype(buf: Any) -> DataType:
    if type(buf).__module__.startswith("torch"):
        import torch
        table = {torch.float32: DataType.FLOAT32, torch.float64: DataType.FLOAT64, torch.int32: DataType.INT32,
                 torch.int64: DataType.INT64, torch.bfloat16: DataType.BF16, torch.float16: DataType.FP16}
    else:
        import numpy as np
        table = {np.dtype(np.float32): DataType.FLOAT32, np.dtype(np.float64): DataType.FLOAT64,
                 np.dtype(np.int32): DataType.INT32, np.dtype(np.int64): DataType.INT64,
                 np.dtype(np.float16): DataType.FP16}
    if buf.dtype not in table:
        raise TypeError(f"unsupported dtype {buf.dtype}")
    return table[buf.dtype]


def _dtype_of(buf: Any) -> DataType:
    # Per-call path of every collective: one dict lookup once a dtype has been seen.
    dt = buf.dtype
    v = _DTYPE_CACHE.get(dt)
    if v is None:
        v = _DTYPE_CACHE[dt] = _resolve_dtype(buf)
    return v


def _ptr(buf: Any) -> Optional[int]:
    if buf is None:
        return None
    data_ptr = getattr(buf, "data_ptr", None)  # torch tensors
    if data_ptr is not None:
        if not buf.is_contiguous():
            raise ValueError("tensors must be contiguous")
        return data_ptr()
    if not buf.flags["C_CONTIGUOUS"]:
        raise ValueError("arrays must be C-contiguous")
    return buf.ctypes.data


def _numel(buf: Any) -> int:
    numel = getattr(buf, "numel", None)
    if callable(numel):
        return numel()
    return int(buf.size)


def _nbytes(buf: Any) -> int:
    if type(buf).__module__.startswith("torch"):
        return buf.numel() * buf.element_size()
    return int(buf.nbytes)


_RAW_STREAM = None


def _current_raw_stream(device: int) -> int:
    """The current torch CUDA stream of ``device`` as a raw handle (without building a Stream
    object on every call)."""
    global _RAW_STREAM
    if _RAW_STREAM is None:
        import torch
        raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
        _RAW_STREAM = raw if raw is not None else (lambda d: torch.cuda.current_stream(d).cuda_stream)
    return int(_RAW_STREAM(device))


class Communicator:
    """One rank's communicator (see module docstring)."""

    def __init__(self) -> None:
        self._lib = _native.lib()
        h = ctypes.c_void_p()
        self._check(self._lib.bcclCommCreate(ctypes.byref(h)))
        self._h = h
        self._inited = False
        self.device: int = -1
        self.blocking = False

    # ---------------------------------------------------------------- lifecycle
    def _check(self, rc: int) -> None:
        if rc != 0:
            raise BcclError(_native.last_error() or "bccl call failed")

    def get_unique_id(self) -> UniqueId:
        ip = ctypes.create_string_buffer(64)
        port = ctypes.c_uint16()
        self._check(self._lib.bcclGetUniqueId(self._h, ip, ctypes.byref(port)))
        return UniqueId(ip.value.decode(), port.value)

    def init(self, rank: int, world_size: int, unique_id: Optional[UniqueId] = None, *, device: int = -1,
             n_channels: int = 0, buffer_bytes: int = 0, timeout_ms: int = 0, enable_nvls: bool = True,
             enable_nccl_p2p: bool = True, logical_machine_size: int = 0, blocking: bool = False) -> "Communicator":
        cfg = _native.BcclConfig()
        cfg.rank, cfg.world_size = rank, world_size
        uid = unique_id or UniqueId("127.0.0.1", 0)
        cfg.ip_addr = uid.ip_addr.encode()
        cfg.port = uid.port
        cfg.n_channels = n_channels
        cfg.device = device
        cfg.buffer_bytes = buffer_bytes
        cfg.timeout_ms = timeout_ms
        cfg.enable_nvls = int(enable_nvls)
        cfg.enable_nccl_p2p = int(enable_nccl_p2p)
        cfg.logical_machine_size = logical_machine_size
        self._check(self._lib.bcclCommInit(self._h, ctypes.byref(cfg)))
        self._inited = True
        self.device = device
        self.blocking = blocking
        return self

    def split(self, color: int, key: Optional[int] = None) -> Optional["Communicator"]:
        """Collective: the ranks passing the same ``color`` >= 0 form a new communicator, ranked
        by (``key``, rank) (``key`` defaults to this rank); ``color`` < 0 returns None. The new
        communicator has the same kind (device or host), channels and timeouts."""
        out = ctypes.c_void_p()
        self._check(self._lib.bcclCommSplit(self._h, int(color), int(self.rank if key is None else key),
                                            ctypes.byref(out)))
        if not out.value:
            return None
        child = Communicator.__new__(Communicator)
        child._lib = self._lib
        child._h = out
        child._inited = True
        child.device = self.device
        child.blocking = self.blocking
        return child

    def finalize(self) -> None:
        if self._h is not None:
            self._lib.bcclCommFinalize(self._h)
            self._inited = False

    def destroy(self) -> None:
        if self._h is not None:
            self._lib.bcclCommFinalize(self._h)
            self._lib.bcclCommDestroy(self._h)
            self._h = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order varies
        try:
            self.destroy()
        except Exception:
            pass

    # ---------------------------------------------------------------- views
    def _info(self) -> tuple:
        vals = [ctypes.c_int() for _ in range(7)]
        self._check(self._lib.bcclCommInfo(self._h, *[ctypes.byref(v) for v in vals]))
        return tuple(v.value for v in vals)

    @property
    def rank(self) -> int:
        return self._info()[0]

    @property
    def world_size(self) -> int:
        return self._info()[1]

    @property
    def local_rank(self) -> int:
        return self._info()[2]

    @property
    def local_size(self) -> int:
        return self._info()[3]

    @property
    def machine_index(self) -> int:
        return self._info()[4]

    @property
    def machine_count(self) -> int:
        return self._info()[5]

    @property
    def n_channels(self) -> int:
        return self._info()[6]

    @property
    def is_single_machine(self) -> bool:
        return self.machine_count == 1

    def _int_list(self, fn) -> list:
        buf = (ctypes.c_int * 256)()
        n = fn(self._h, buf, 256)
        return [buf[i] for i in range(min(n, 256))]

    @property
    def local_ranks(self) -> list:
        return self._int_list(self._lib.bcclCommLocalRanks)

    @property
    def machine_leaders(self) -> list:
        return self._int_list(self._lib.bcclCommMachineLeaders)

    @property
    def nvls_enabled(self) -> bool:
        return bool(self._lib.bcclCommNvlsEnabled(self._h))

    @property
    def last_algorithm(self) -> str:
        return self._lib.bcclCommLastAlgorithm(self._h).decode()

    @property
    def kernel_launches(self) -> int:
        return int(self._lib.bcclCommKernelLaunches(self._h))

    def p2p_transport(self, peer: int) -> str:
        return self._lib.bcclCommP2pTransport(self._h, peer).decode()

    @property
    def host_executor(self) -> str:
        return self._lib.bcclCommHostExecutor(self._h).decode()

    @property
    def host_zero_copy(self) -> tuple:
        """(enabled, messages received): single-copy Send/Recv between ranks of one machine
        (host communicators; messages of at least BCCL_HOST_ZC_BYTES, default 256 KiB)."""
        en = ctypes.c_int(0)
        n = int(self._lib.bcclCommHostZeroCopyTransfers(self._h, ctypes.byref(en)))
        return bool(en.value), n

    # ---------------------------------------------------------------- streams
    def _stream(self, stream: Any = None) -> tuple:
        if self.device < 0:
            return 0, 0
        if self.blocking and stream is None:
            import torch
            if torch.cuda.is_current_stream_capturing():
                raise BcclError("a blocking communicator runs on its own stream and waits on the host, so it "
                                "cannot be captured into a CUDA graph; use a stream-ordered one (blocking=False)")
            # The library's stream is ordered after the legacy default stream only; torch may have
            # written the inputs on another stream of this device.
            cur = torch.cuda.current_stream(self.device)
            if cur.cuda_stream != 0:
                cur.synchronize()
            return 0, 0
        if stream is None:
            return _current_raw_stream(self.device), 1
        handle = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
        return int(handle), 1

    # ---------------------------------------------------------------- argument checks
    # On the per-call path of every collective: a few attribute reads for torch tensors.
    def _where(self, t: Any) -> None:
        """t must live where this communicator's kernels or threads can address it: device
        memory for a device communicator, host memory for a host one (a pointer of the other
        kind would be dereferenced by a kernel or by memcpy)."""
        on_gpu = getattr(t, "is_cuda", False)
        if on_gpu is not (self.device >= 0):
            raise ValueError(f"bccl: a {'device' if self.device >= 0 else 'host'} communicator got a "
                             f"{'CUDA' if on_gpu else 'host'} buffer")

    def _pair(self, name: str, a: Any, b: Any, nb: int) -> None:
        """a is in this communicator's memory; b (unless None or a itself: in place) too, with
        a's dtype and nb elements."""
        gpu = self.device >= 0
        try:  # torch tensors: five attribute reads when everything matches
            if a.is_cuda is gpu and (b is None or b is a or
                                     (b.is_cuda is gpu and b.dtype == a.dtype and b.numel() == nb)):
                return
        except AttributeError:  # numpy arrays (host memory)
            pass
        self._where(a)
        if b is None or b is a:
            return
        self._where(b)
        if b.dtype != a.dtype or _numel(b) != nb:
            raise ValueError(f"bccl: {name}: the other buffer needs {nb} elements of dtype {a.dtype}, got "
                             f"{_numel(b)} of {b.dtype}")

    # ---------------------------------------------------------------- collectives
    def all_reduce(self, tensor: Any, op: ReduceOp = ReduceOp.SUM, *, out: Any = None, scale: float = 1.0,
                   algo: Algo = Algo.AUTO, stream: Any = None) -> Any:
        """out = reduce(tensor over ranks) * scale; in place when ``out`` is None."""
        out = tensor if out is None else out
        n = _numel(tensor)
        self._pair("all_reduce", tensor, out, n)
        s, has = self._stream(stream)
        # DataType / ReduceOp / Algo are IntEnums: ctypes takes them as ints.
        src = _ptr(tensor)
        self._check(self._lib.bcclAllReduce(self._h, src, src if out is tensor else _ptr(out), n, _dtype_of(tensor),
                                            op, float(scale), algo, s, has))
        return out

    def broadcast(self, tensor: Any, root: int, *, src: Any = None, algo: Algo = Algo.AUTO, stream: Any = None) -> Any:
        """Every rank's ``tensor`` receives the root's data (``src`` on the root when out of place)."""
        n = _numel(tensor)
        self._pair("broadcast", tensor, src, n)
        s, has = self._stream(stream)
        self._check(self._lib.bcclBroadcast(self._h, _ptr(src) if src is not None else _ptr(tensor), _ptr(tensor),
                                            _numel(tensor), int(_dtype_of(tensor)), int(root), int(algo), s, has))
        return tensor

    def reduce(self, tensor: Any, root: int, op: ReduceOp = ReduceOp.SUM, *, out: Any = None, algo: Algo = Algo.AUTO,
               stream: Any = None) -> Any:
        """The root's ``out`` (default: ``tensor``) receives the reduction; other ranks' out may be None."""
        dst = out if out is not None else (tensor if self.rank == root else None)
        n = _numel(tensor)
        self._pair("reduce", tensor, dst, n)
        s, has = self._stream(stream)
        self._check(self._lib.bcclReduce(self._h, _ptr(tensor), _ptr(dst), _numel(tensor), int(_dtype_of(tensor)),
                                         int(op), int(root), int(algo), s, has))
        return dst

    def all_gather(self, out: Any, tensor: Any, *, algo: Algo = Algo.AUTO, stream: Any = None) -> Any:
        """out (world_size * numel) = concatenation of every rank's tensor in rank order."""
        n = _numel(tensor)
        self._pair("all_gather", tensor, out, n * self.world_size)
        s, has = self._stream(stream)
        self._check(self._lib.bcclAllGatherAlgo(self._h, _ptr(tensor), _ptr(out), n, _dtype_of(tensor), algo, s, has))
        return out

    def reduce_scatter(self, out: Any, tensor: Any, op: ReduceOp = ReduceOp.SUM, *, algo: Algo = Algo.AUTO,
                       stream: Any = None) -> Any:
        """out (numel) = this rank's block of reduce(tensor (world_size * numel))."""
        n = _numel(out)
        self._pair("reduce_scatter", out, tensor, n * self.world_size)
        s, has = self._stream(stream)
        self._check(self._lib.bcclReduceScatterAlgo(self._h, _ptr(tensor), _ptr(out), n, _dtype_of(out), op, algo,
                                                    s, has))
        return out

    def send(self, tensor: Any, peer: int, *, stream: Any = None) -> None:
        self._where(tensor)
        s, has = self._stream(stream)
        self._check(self._lib.bcclSend(self._h, _ptr(tensor), _numel(tensor), int(_dtype_of(tensor)), int(peer), s, has))

    def recv(self, tensor: Any, peer: int, *, stream: Any = None) -> Any:
        self._where(tensor)
        s, has = self._stream(stream)
        self._check(self._lib.bcclRecv(self._h, _ptr(tensor), _numel(tensor), int(_dtype_of(tensor)), int(peer), s, has))
        return tensor

    def all_to_all(self, out: Any, tensor: Any, *, stream: Any = None) -> Any:
        """out block q = block `rank` of rank q's tensor, where tensor and out (both contiguous,
        world_size * n elements) are cut into world_size blocks of n: the exchange behind
        expert-parallel dispatch and combine. One group of Send/Recv with every peer (on a device
        communicator with BCCL_P2P_NATIVE=1 that is one kernel launch); the own block is copied
        locally. The reference has no AllToAll (its collectives are the five of
        OriginCCL include/types.h:30-38); this composes its Send/Recv semantics."""
        w, r = self.world_size, self.rank
        total = _numel(tensor)
        if total % w != 0 or _numel(out) != total:
            raise ValueError(f"all_to_all: tensor and out need world_size * n elements (got {total}, {_numel(out)})")
        n = total // w
        t, o = tensor.reshape(-1), out.reshape(-1)
        o[r * n:(r + 1) * n] = t[r * n:(r + 1) * n]
        if w > 1 and n > 0:
            with self.group(stream):
                for q in range(w):
                    if q != r:
                        self.send(t[q * n:(q + 1) * n], q, stream=stream)
                        self.recv(o[q * n:(q + 1) * n], q, stream=stream)
        return out

    def batch(self, tensors: Sequence[Any], outs: Optional[Sequence[Any]] = None) -> "TensorBatch":
        """Pointer arrays for :meth:`all_reduce_many`, built once for tensors that are synced often."""
        return TensorBatch(tensors, outs)

    def all_reduce_many(self, tensors: Any, op: ReduceOp = ReduceOp.SUM, *, scale: float = 1.0,
                        grouped: bool = True, stream: Any = None) -> None:
        """AllReduce of every tensor (in place, or into the batch's outputs) in ONE library call.

        ``tensors`` is a list of same-dtype tensors or a :class:`TensorBatch`. With ``grouped`` the
        calls form one GroupStart/GroupEnd batch (small tensors then run as one kernel); without,
        each runs as its own operation in order.
        """
        b = tensors if isinstance(tensors, TensorBatch) else TensorBatch(tensors)
        s, has = self._stream(stream)
        self._check(self._lib.bcclAllReduceMany(self._h, b.n, b.send, b.recv, b.counts, int(b.dtype), int(op),
                                                float(scale), int(grouped), s, has))

    # Raw-pointer entry points (device pointers or host addresses), for callers without tensors.
    def all_reduce_ptr(self, send: int, recv: int, count: int, dtype: DataType, op: ReduceOp = ReduceOp.SUM,
                       scale: float = 1.0, algo: Algo = Algo.AUTO, stream: Any = None) -> None:
        s, has = self._stream(stream)
        self._check(self._lib.bcclAllReduce(self._h, send, recv, count, int(dtype), int(op), float(scale), int(algo),
                                            s, has))

    # ---------------------------------------------------------------- groups
    def group_start(self) -> None:
        self._check(self._lib.bcclGroupStart(self._h))

    def group_end(self, stream: Any = None) -> None:
        s, has = self._stream(stream)
        self._check(self._lib.bcclGroupEnd(self._h, s, has))

    @contextlib.contextmanager
    def group(self, stream: Any = None):
        self.group_start()
        ok = False
        try:
            yield self
            ok = True
        finally:
            if ok:
                self.group_end(stream)
            else:
                # Leave the group without hiding the original exception.
                try:
                    self.group_end(stream)
                except BcclError:
                    pass

    # ---------------------------------------------------------------- misc
    def async_error(self) -> int:
        """Without synchronising: 0, or the failure a device kernel has recorded so far (1 timeout,
        2 aborted, 3 bad arguments); 1 after a failed host operation. For CUDA-graph replays and
        other stream-ordered use, where no library call returns the error."""
        code = ctypes.c_int(0)
        self._check(self._lib.bcclCommGetAsyncError(self._h, ctypes.byref(code)))
        return code.value

    def synchronize(self) -> None:
        self._check(self._lib.bcclSynchronize(self._h))

    def device_state(self) -> tuple:
        """Device communicators: the device-side sequence counters after the queued work (round,
        barrier, NVLS round, ring message, fused-TP launch, finished CTAs of the current launch).
        Every rank holds the same values after the same calls; synchronises the device."""
        out = (ctypes.c_ulonglong * 6)()
        if self._lib.bcclDebugDeviceState(self._h, out) != 0:
            raise BcclError("device state unavailable (not a device communicator?)")
        return tuple(int(v) for v in out)

    def dump_trace(self, path: str) -> int:
        """Writes the trace recorded since the last dump (BCCL_TRACE=<records> at init) as
        Chrome-trace JSON: per-CTA kernel events on device communicators, per-channel phases
        (copy-in, barrier waits, reduction, leader exchange, copy-out) on host ones. Returns
        the number of events, -1 when tracing is off."""
        return int(self._lib.bcclTraceDump(self._h, path.encode()))

    def abort(self) -> None:
        """Stops the operations in flight (callable from another thread): host waits return at
        once, device waits within ~1 ms; the operation raises. Only destroy() is useful after."""
        self._lib.bcclCommAbort(self._h)

    def barrier(self) -> None:
        """Host-side barrier over the bootstrap (no device work)."""
        self._check(self._lib.bcclBarrier(self._h))

    def symmetric_empty(self, shape: Sequence[int], dtype: Any) -> Any:
        """Collective: a CUDA tensor in memory every rank can address (freed with the communicator)."""
        import torch
        numel = 1
        for d in shape:
            numel *= int(d)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        ptr = self._lib.bcclSymmetricAlloc(self._h, max(nbytes, 1))
        if not ptr:
            raise BcclError(_native.last_error() or "symmetric allocation failed")
        return _tensor_from_ptr(ptr, shape, dtype, self.device)

    def register(self, tensor: Any) -> Any:
        """Collective: lets the peers address ``tensor``'s memory (CUDA IPC) so that AllReduce,
        AllGather and ReduceScatter of at least 1 MiB on it (or on a view at the same offset on
        every rank) run without staging copies. Every rank registers its own tensor of the same
        size, in the same order. Each rank decides from its own registrations whether a call runs
        zero-copy, so a call's buffers must be registered on every rank or on none: deregister
        before the memory is freed or reused by other tensors (PyTorch's caching allocator hands
        freed blocks to new tensors, whose collectives would otherwise count as registered on this
        rank only). Host communicators ignore it. Returns ``tensor``."""
        self._check(self._lib.bcclCommRegister(self._h, _ptr(tensor), _nbytes(tensor)))
        return tensor

    def deregister(self, tensor: Any) -> None:
        """Collective: undoes ``register`` (waits for the device and for every rank)."""
        self._check(self._lib.bcclCommDeregister(self._h, _ptr(tensor)))

    @contextlib.contextmanager
    def registered(self, *tensors: Any):
        """``with comm.registered(a, b): ...`` registers the tensors for the block."""
        done = []
        try:
            for t in tensors:
                done.append(self.register(t))
            yield tensors
        finally:
            for t in reversed(done):
                self.deregister(t)


class TensorBatch:
    """Send/recv pointer and count arrays of many same-dtype tensors (see Communicator.batch)."""

    def __init__(self, tensors: Sequence[Any], outs: Optional[Sequence[Any]] = None) -> None:
        tensors = list(tensors)
        outs = tensors if outs is None else list(outs)
        if len(outs) != len(tensors):
            raise ValueError("outs must match tensors")
        self.n = len(tensors)
        self.dtype = _dtype_of(tensors[0]) if tensors else DataType.FLOAT32
        for t in tensors:
            if _dtype_of(t) != self.dtype:
                raise TypeError("all tensors of a batch must have one dtype")
        self.send = (ctypes.c_void_p * max(self.n, 1))(*[_ptr(t) for t in tensors])
        self.recv = (ctypes.c_void_p * max(self.n, 1))(*[_ptr(t) for t in outs])
        self.counts = (ctypes.c_size_t * max(self.n, 1))(*[_numel(t) for t in tensors])
        self._keep = (tensors, outs)  # the pointers stay valid while the batch lives


def _tensor_from_ptr(ptr: int, shape: Sequence[int], dtype: Any, device: int) -> Any:
    import torch

    class _Holder:
        __cuda_array_interface__ = None

    typestr = {torch.float32: "<f4", torch.float64: "<f8", torch.int32: "<i4", torch.int64: "<i8",
               torch.float16: "<f2", torch.bfloat16: "<f2", torch.uint8: "|u1"}[dtype]
    h = _Holder()
    h.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr, "data": (ptr, False),
                                  "version": 3}
    with torch.cuda.device(device):
        t = torch.as_tensor(h, device=f"cuda:{device}")
    if dtype == torch.bfloat16:
        t = t.view(torch.bfloat16)
    return t


# ---------------------------------------------------------------- bootstrapping helpers

_STORE_KEY_USES: dict = {}


def init_from_store(store: Any, rank: int, world_size: int, *, key: str = "bccl_uid", **kwargs) -> Communicator:
    """Creates a communicator, distributing the unique id through a torch.distributed Store.

    Collective over the ranks. Each call with the same ``store`` and ``key`` in a process uses a
    fresh store entry (``key``, ``key.1``, ``key.2``, ...), so ranks that create several
    communicators on one store in the same order never read an earlier communicator's id."""
    uses = (id(store), key)
    n = _STORE_KEY_USES.get(uses, 0)
    _STORE_KEY_USES[uses] = n + 1
    key = key if n == 0 else f"{key}.{n}"
    comm = Communicator()
    if rank == 0:
        uid = comm.get_unique_id()
        store.set(key, uid.to_bytes())
    else:
        uid = UniqueId.from_bytes(store.get(key))
    return comm.init(rank, world_size, uid, **kwargs)


def init_from_env(**kwargs) -> Communicator:
    """Creates a communicator from the launcher's environment.

    ``bccl_run`` exports BCCL_RANK / BCCL_WORLD_SIZE / BCCL_ID_FILE (rank 0 writes the unique
    id to the file, the others wait for it), or, across nodes, BCCL_MASTER=<addr>:<port> (rank 0
    listens there, the others connect to it). Under torchrun (RANK / WORLD_SIZE set) the id goes
    through the default torch.distributed store when a process group exists.
    """
    if "BCCL_RANK" in os.environ:
        rank, world = int(os.environ["BCCL_RANK"]), int(os.environ["BCCL_WORLD_SIZE"])
        if "device" not in kwargs and "BCCL_DEVICE" in os.environ:  # bccl_run --gpus
            kwargs["device"] = int(os.environ["BCCL_DEVICE"])
        comm = Communicator()
        master = os.environ.get("BCCL_MASTER")  # multi-node launch: rank 0 listens there
        if master:
            uid = comm.get_unique_id() if rank == 0 else UniqueId.from_bytes(master.encode())
            return comm.init(rank, world, uid, **kwargs)
        path = os.environ["BCCL_ID_FILE"]
        if rank == 0:
            uid = comm.get_unique_id()
            tmp = path + ".tmp"
            with open(tmp, "wb") as f:
                f.write(uid.to_bytes())
            os.replace(tmp, path)
        else:
            deadline = time.time() + 60
            while not os.path.exists(path):
                if time.time() > deadline:
                    raise BcclError("timed out waiting for the unique id file")
                time.sleep(0.01)
            with open(path, "rb") as f:
                uid = UniqueId.from_bytes(f.read())
        return comm.init(rank, world, uid, **kwargs)
    import torch.distributed as dist
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    if world == 1:
        return Communicator().init(0, 1, None, **kwargs)
    if not dist.is_initialized():
        raise BcclError("init_from_env under torchrun needs torch.distributed.init_process_group first")
    store = dist.distributed_c10d._get_default_store()
    return init_from_store(store, rank, world, **kwargs)
