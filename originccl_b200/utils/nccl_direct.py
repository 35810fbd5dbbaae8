"""NCCL called directly (ctypes), for same-op comparisons in the benchmarks.

torch.distributed only exposes in-place AllReduce. The comparison arm of ``bench.py`` and
``utils.sweep`` must run the same operation as this library — out of place on the same rotating
inputs, or in place — so this module opens the NCCL that torch already loaded (``libnccl.so.2``,
or ``BCCL_NCCL_LIBRARY``), creates one NCCL communicator per process with its unique id passed
through a torch.distributed store, and calls ``ncclAllReduce`` / ``ncclReduceScatter`` /
``ncclAllGather`` / ``ncclBroadcast`` / ``ncclReduce`` on torch tensors and the current stream.
"""
from __future__ import annotations

import ctypes
import os
from typing import Any

_DTYPES = {"int32": 2, "int64": 4, "float16": 6, "float32": 7, "float64": 8, "bfloat16": 9}
_OPS = {"sum": 0, "prod": 1, "max": 2, "min": 3, "avg": 4}


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]


def _dtype_code(t: Any) -> int:
    name = str(t.dtype).replace("torch.", "")
    if name not in _DTYPES:
        raise ValueError(f"NCCL comparison: unsupported dtype {name}")
    return _DTYPES[name]


class NcclDirect:
    """One NCCL communicator over all ranks of the job (collective constructor)."""

    _instances = 0

    def __init__(self, store: Any, rank: int, world: int, device: int, tag: str = "") -> None:
        import torch
        self.lib = ctypes.CDLL(os.environ.get("BCCL_NCCL_LIBRARY", "libnccl.so.2"), mode=ctypes.RTLD_GLOBAL)
        self.rank, self.world, self.device = rank, world, device
        key = f"bccl_nccl_direct_uid_{tag}_{NcclDirect._instances}"
        NcclDirect._instances += 1
        uid = _UniqueId()
        if rank == 0:
            self._ok(self.lib.ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
            # All 128 bytes: reading the c_char array field would stop at its first zero byte.
            store.set(key, ctypes.string_at(ctypes.addressof(uid), ctypes.sizeof(uid)))
        else:
            raw = store.get(key)
            ctypes.memmove(ctypes.byref(uid), raw, 128)
        torch.cuda.set_device(device)
        self.comm = ctypes.c_void_p()
        self._ok(self.lib.ncclCommInitRank(ctypes.byref(self.comm), ctypes.c_int(world), uid, ctypes.c_int(rank)),
                 "ncclCommInitRank")

    def _ok(self, rc: int, what: str) -> None:
        if rc != 0:
            self.lib.ncclGetErrorString.restype = ctypes.c_char_p
            raise RuntimeError(f"{what} failed: {self.lib.ncclGetErrorString(rc).decode()}")

    @staticmethod
    def _stream(device: int) -> ctypes.c_void_p:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)

    def all_reduce(self, send: Any, recv: Any, op: str = "sum") -> None:
        self._ok(self.lib.ncclAllReduce(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                                        ctypes.c_size_t(send.numel()), _dtype_code(send), _OPS[op], self.comm,
                                        self._stream(self.device)), "ncclAllReduce")

    def reduce_scatter(self, send: Any, recv: Any, op: str = "sum") -> None:
        self._ok(self.lib.ncclReduceScatter(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                                            ctypes.c_size_t(recv.numel()), _dtype_code(send), _OPS[op], self.comm,
                                            self._stream(self.device)), "ncclReduceScatter")

    def all_gather(self, send: Any, recv: Any) -> None:
        self._ok(self.lib.ncclAllGather(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                                        ctypes.c_size_t(send.numel()), _dtype_code(send), self.comm,
                                        self._stream(self.device)), "ncclAllGather")

    def broadcast(self, send: Any, recv: Any, root: int) -> None:
        self._ok(self.lib.ncclBroadcast(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                                        ctypes.c_size_t(recv.numel()), _dtype_code(recv), ctypes.c_int(root),
                                        self.comm, self._stream(self.device)), "ncclBroadcast")

    def reduce(self, send: Any, recv: Any, root: int, op: str = "sum") -> None:
        self._ok(self.lib.ncclReduce(ctypes.c_void_p(send.data_ptr()), ctypes.c_void_p(recv.data_ptr()),
                                     ctypes.c_size_t(send.numel()), _dtype_code(send), _OPS[op], ctypes.c_int(root),
                                     self.comm, self._stream(self.device)), "ncclReduce")

    def destroy(self) -> None:
        if self.comm:
            self.lib.ncclCommDestroy(self.comm)
            self.comm = ctypes.c_void_p()
