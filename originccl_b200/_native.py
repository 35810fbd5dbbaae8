"""ctypes binding of the native library's C interface (csrc/include/bccl/c_api.h).

The library is loaded from ``originccl_b200/_lib/libbccl.so`` in the source tree (built by
``originccl_b200._build``); it is never looked up elsewhere, so the code that runs is the code
in this repository. If it is missing, importing this module raises instead of falling back.
"""
from __future__ import annotations

import ctypes
import os
import sysconfig
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libbccl.so"


class BcclConfig(ctypes.Structure):
    _fields_ = [
        ("rank", ctypes.c_int),
        ("world_size", ctypes.c_int),
        ("ip_addr", ctypes.c_char * 64),
        ("port", ctypes.c_uint16),
        ("n_channels", ctypes.c_int),
        ("device", ctypes.c_int),
        ("buffer_bytes", ctypes.c_size_t),
        ("timeout_ms", ctypes.c_int),
        ("enable_nvls", ctypes.c_int),
        ("enable_nccl_p2p", ctypes.c_int),
        ("logical_machine_size", ctypes.c_int),
    ]


def _point_at_nccl() -> None:
    """The device communicator dlopens libnccl.so.2 for Send/Recv; prefer PyTorch's copy."""
    if os.environ.get("BCCL_NCCL_LIBRARY"):
        return
    p = Path(sysconfig.get_paths()["purelib"]) / "nvidia" / "nccl" / "lib" / "libnccl.so.2"
    if p.exists():
        os.environ["BCCL_NCCL_LIBRARY"] = str(p)


def load(path: Path | None = None) -> ctypes.CDLL:
    path = Path(path) if path else _LIB_PATH
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build the native library first "
            "(python -c 'import __graft_entry__ as g; g.build()' or python -m originccl_b200._build)")
    _point_at_nccl()
    lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
    c_int, c_size, vp, u64 = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint64
    up = ctypes.c_size_t  # uintptr_t
    sig = {
        "bcclCommCreate": (c_int, [ctypes.POINTER(vp)]),
        "bcclGetUniqueId": (c_int, [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint16)]),
        "bcclCommInit": (c_int, [vp, ctypes.POINTER(BcclConfig)]),
        "bcclCommFinalize": (c_int, [vp]),
        "bcclCommDestroy": (c_int, [vp]),
        "bcclCommGetAsyncError": (c_int, [vp, ctypes.POINTER(c_int)]),
        "bcclCommSplit": (c_int, [vp, c_int, c_int, ctypes.POINTER(vp)]),
        "bcclGetLastError": (ctypes.c_char_p, []),
        "bcclVersion": (ctypes.c_char_p, []),
        "bcclCommInfo": (c_int, [vp] + [ctypes.POINTER(c_int)] * 7),
        "bcclCommLocalRanks": (c_int, [vp, ctypes.POINTER(c_int), c_int]),
        "bcclCommMachineLeaders": (c_int, [vp, ctypes.POINTER(c_int), c_int]),
        "bcclCommNvlsEnabled": (c_int, [vp]),
        "bcclCommLastAlgorithm": (ctypes.c_char_p, [vp]),
        "bcclCommKernelLaunches": (ctypes.c_ulonglong, [vp]),
        "bcclCommP2pTransport": (ctypes.c_char_p, [vp, c_int]),
        "bcclCommHostExecutor": (ctypes.c_char_p, [vp]),
        "bcclCommHostZeroCopyTransfers": (ctypes.c_ulonglong, [vp, ctypes.POINTER(c_int)]),
        "bcclGroupStart": (c_int, [vp]),
        "bcclGroupEnd": (c_int, [vp, up, c_int]),
        "bcclAllReduce": (c_int, [vp, vp, vp, c_size, c_int, c_int, ctypes.c_float, c_int, up, c_int]),
        "bcclAllReduceMany": (c_int, [vp, c_int, vp, vp, vp, c_int, c_int, ctypes.c_float, c_int, up, c_int]),
        "bcclBroadcast": (c_int, [vp, vp, vp, c_size, c_int, c_int, c_int, up, c_int]),
        "bcclReduce": (c_int, [vp, vp, vp, c_size, c_int, c_int, c_int, c_int, up, c_int]),
        "bcclAllGather": (c_int, [vp, vp, vp, c_size, c_int, up, c_int]),
        "bcclReduceScatter": (c_int, [vp, vp, vp, c_size, c_int, c_int, up, c_int]),
        "bcclAllGatherAlgo": (c_int, [vp, vp, vp, c_size, c_int, c_int, up, c_int]),
        "bcclReduceScatterAlgo": (c_int, [vp, vp, vp, c_size, c_int, c_int, c_int, up, c_int]),
        "bcclSend": (c_int, [vp, vp, c_size, c_int, c_int, up, c_int]),
        "bcclRecv": (c_int, [vp, vp, c_size, c_int, c_int, up, c_int]),
        "bcclSynchronize": (c_int, [vp]),
        "bcclBarrier": (c_int, [vp]),
        "bcclSymmetricAlloc": (vp, [vp, c_size]),
        "bcclSymmetricFree": (c_int, [vp, vp]),
        "bcclCommRegister": (c_int, [vp, vp, c_size]),
        "bcclCommDeregister": (c_int, [vp, vp]),
        "bcclPlannerSort": (c_int, [c_int, c_int, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_size),
                                    ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                    ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
        "bcclDebugWaitProbe": (c_int, [vp, c_int]),
        "bcclDebugDeviceState": (c_int, [vp, ctypes.POINTER(ctypes.c_ulonglong)]),
        "bcclGemmBf16": (c_int, [vp, vp, vp, c_int, c_int, c_int, c_int, c_int, vp]),
        "bcclGemmCheckError": (c_int, []),
        "bcclGemmUsesPair": (c_int, []),
        "bcclGemmTileWidth": (c_int, [c_int, c_int]),
        "bcclCommAbort": (c_int, [vp]),
        "bcclTpAllGatherGemm": (c_int, [vp, vp, vp, vp, c_int, c_int, c_int, c_int, up, c_int]),
        "bcclTpGemmReduceScatter": (c_int, [vp, vp, vp, vp, c_int, c_int, c_int, up, c_int]),
        "bcclTraceDump": (ctypes.c_long, [vp, ctypes.c_char_p]),
        "bcclDebugBandwidth": (ctypes.c_double, [vp, c_int, c_int, c_size, c_int, c_int]),
        "bcclPlannerP2pRound": (c_int, [c_int, c_int, c_int, c_int]),
        "bcclP2pChannels": (c_int, [ctypes.c_ulonglong]),
        "bcclLLEpoch": (ctypes.c_uint, [ctypes.c_ulonglong]),
        "bcclP2pPlan": (c_int, [ctypes.POINTER(ctypes.c_ulonglong), c_int, c_int, c_int, c_int, ctypes.POINTER(c_int),
                                ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(ctypes.c_ulonglong)]),
        "bcclPlannerValidate": (c_int, [c_int, c_int, c_int, c_size, c_int, c_int, c_int, c_int, c_int, c_int]),
        "bcclPlannerChoose": (c_int, [c_int, c_int, c_int, c_size, c_int, c_int, c_int, ctypes.POINTER(c_int),
                                      ctypes.POINTER(c_int)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del u64
    return lib


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def last_error() -> str:
    msg = lib().bcclGetLastError()
    return msg.decode() if msg else ""
