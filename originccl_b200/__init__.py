"""originccl_b200: a Blackwell-native (sm_100a) collective communication library.

The native core (``originccl_b200/_lib/libbccl.so``) is C++/CUDA: a TCP bootstrap, a planner, a
host-memory engine (shared memory + TCP) and a device engine whose collectives are hand-written
sm_100a kernels over NVLink peer memory and NVSwitch multicast. Python reaches it through the C
interface; see :mod:`originccl_b200.comm` for the API.
"""
from .comm import (Algo, BcclError, CollFunc, Communicator, DataType, ReduceOp, UniqueId, init_from_env,
                   init_from_store)

__all__ = ["Algo", "BcclError", "CollFunc", "Communicator", "DataType", "ReduceOp", "UniqueId", "init_from_env",
           "init_from_store", "version"]


def version() -> str:
    from . import _native
    return _native.lib().bcclVersion().decode()
