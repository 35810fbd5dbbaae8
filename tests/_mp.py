"""Runs a function on N spawned rank processes that share a communicator unique id."""
from __future__ import annotations

import multiprocessing as mp
import os
import tempfile
import traceback
from typing import Any, Callable, Dict, List, Optional


def _entry(rank: int, world: int, idfile: str, fn: Callable, args: tuple, q: Any, env: Dict[str, str]) -> None:
    os.environ.update(env)
    os.environ.update(BCCL_RANK=str(rank), BCCL_WORLD_SIZE=str(world), BCCL_ID_FILE=idfile)
    try:
        q.put((rank, True, fn(rank, world, *args)))
    except BaseException:  # report everything, including assertion failures
        q.put((rank, False, traceback.format_exc()))


def run(world: int, fn: Callable, *args: Any, timeout: float = 120.0, env: Optional[Dict[str, str]] = None,
        expect_fail: bool = False) -> List[Any]:
    """Returns the per-rank results in rank order; raises if any rank failed (unless expect_fail,
    in which case the per-rank (ok, result) pairs are returned)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    d = tempfile.mkdtemp(prefix="bccl-test-")
    idfile = os.path.join(d, "uid")
    procs = [ctx.Process(target=_entry, args=(r, world, idfile, fn, args, q, env or {})) for r in range(world)]
    for p in procs:
        p.start()
    results: Dict[int, Any] = {}
    try:
        for _ in procs:
            rank, ok, val = q.get(timeout=timeout)
            results[rank] = (ok, val)
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
                p.join()
    if expect_fail:
        return [results.get(r, (False, "no result")) for r in range(world)]
    errors = [f"rank {r}: {v}" for r, (ok, v) in sorted(results.items()) if not ok]
    if errors:
        raise AssertionError("\n".join(errors))
    return [results[r][1] for r in range(world)]
