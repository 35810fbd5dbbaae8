"""Starts N ranks of a command on this machine through the ``bccl_run`` launcher (no MPI).

    python -m originccl_b200.run -np 4 [--gpus] [--timeout SEC] -- python my_script.py args...
    python -m originccl_b200.run -np 8 --nnodes 2 --node-rank K --master ADDR:PORT -- ...   # per node

Each rank gets BCCL_RANK / BCCL_WORLD_SIZE / BCCL_LOCAL_RANK / BCCL_ID_FILE (and BCCL_DEVICE with
``--gpus``); ``originccl_b200.init_from_env()`` picks them up. The exit status is the first failing
rank's, and the other ranks are stopped when one fails.
"""
from __future__ import annotations

import os
import sys


def launcher_path() -> str:
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "bccl_run")
    if not os.path.exists(here):
        from . import _build
        _build.build()
    return here


def main(argv=None) -> int:
    args = list(sys.argv[1:] if argv is None else argv)
    if not args or args[0] in ("-h", "--help"):
        print(__doc__)
        return 0 if args else 2
    exe = launcher_path()
    os.execv(exe, [exe] + args)
    return 127  # not reached


if __name__ == "__main__":
    sys.exit(main())
