"""Device-trace breakdown of one collective kernel on N GPUs (work vs. cross-rank waits).

Multi-rank kernels cannot be captured under ncu (a capture replays each launch ~40 times, which a
kernel that waits on other GPUs does not survive), so their profile comes from the library's own
device trace: with ``BCCL_TRACE=<records>`` every CTA stamps ``%globaltimer`` when it starts,
when it has issued its share of a pipeline iteration (``staged``), when it passes the iteration's
cross-rank barrier (``barrier``) and when it ends. This tool runs ``--warmup`` untraced calls and
``--traced`` traced calls of one collective, then reports for each rank and traced launch the
kernel's span (first begin to last end over CTAs) and, per iteration, the median and max over
CTAs of the staged and barrier stamps relative to the launch's first begin; plus the CUDA-event
time of the same calls (max over ranks). Run one rank per GPU::

    torchrun --nproc-per-node 8 -m originccl_b200.utils.trace_bench --op allreduce --bytes 128M
    torchrun --nproc-per-node 8 -m originccl_b200.utils.trace_bench \
        --cases "allreduce:128M:nvls,allreduce:128M:hybrid,broadcast:64M,allgather:16M:auto:bfloat16"

A case is ``op:bytes[:algo[:dtype[:buffers]]]``; ``--cases`` runs several in one process.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import tempfile


def summarise(trace: dict) -> list:
    """Per launch (kernel serial): span and per-iteration staged / barrier stamps."""
    by_kernel: dict = {}
    for ev in trace.get("traceEvents", []):
        name = ev["name"].split(" ")[0]
        k = ev["args"]["kernel"]
        by_kernel.setdefault(k, []).append((name, ev["args"]["round"], ev["tid"] // 4, float(ev["ts"])))
    out = []
    for k in sorted(by_kernel):
        evs = by_kernel[k]
        begins = [ts for n, _, _, ts in evs if n == "begin"]
        ends = [ts for n, _, _, ts in evs if n == "end"]
        if not begins or not ends:
            continue
        t0 = min(begins)
        rec = {"kernel": k, "ctas": len(begins), "span_us": round(max(ends) - t0, 2),
               "begin_spread_us": round(max(begins) - t0, 2), "iters": []}
        rounds = sorted({r for n, r, _, _ in evs if n in ("staged", "barrier")})
        for r in rounds:
            st = [ts - t0 for n, rr, _, ts in evs if n == "staged" and rr == r]
            ba = [ts - t0 for n, rr, _, ts in evs if n == "barrier" and rr == r]
            it = {"iter": r}
            if st:
                it.update({"staged_med": round(statistics.median(st), 2), "staged_max": round(max(st), 2)})
            if ba:
                it.update({"barrier_med": round(statistics.median(ba), 2), "barrier_max": round(max(ba), 2)})
            rec["iters"].append(it)
        out.append(rec)
    return out


def trace_case(comm, op: str, nbytes: int, algo_name: str, dtype: str, buffers: str, warmup: int, traced: int,
               barrier) -> dict:
    """Runs one traced case on every rank; returns rank 0's record (None elsewhere)."""
    import torch
    import torch.distributed as dist
    from originccl_b200 import Algo

    rank, world = comm.rank, comm.world_size
    dt = getattr(torch, dtype)
    es = torch.empty((), dtype=dt).element_size()
    n = max(1, nbytes // es)
    algo = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS,
            "ring": Algo.RING, "hybrid": Algo.HYBRID, "ll": Algo.LL}[algo_name]
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    nin = n * world if op == "reducescatter" else n
    nout = n * world if op == "allgather" else n
    alloc = (lambda m: comm.symmetric_empty((m,), dt)) if buffers == "symmetric" and world > 1 else \
        (lambda m: torch.empty(m, device="cuda", dtype=dt))
    x, y = alloc(nin), alloc(nout)
    x.copy_((torch.rand(nin, device="cuda", generator=g) * 2 - 1).to(dt))
    if buffers == "registered" and world > 1:
        comm.register(x)
        comm.register(y)

    def call() -> None:
        if op == "allreduce":
            comm.all_reduce(x, out=y, algo=algo)
        elif op == "broadcast":
            comm.broadcast(y, 0, src=x if rank == 0 else None, algo=algo)
        elif op == "reduce":
            comm.reduce(x, 0, out=y, algo=algo)
        elif op == "allgather":
            comm.all_gather(y, x, algo=algo)
        else:
            comm.reduce_scatter(y, x, algo=algo)

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    path = os.path.join(tempfile.gettempdir(), f"bccl_trace_{os.getpid()}.json")
    comm.dump_trace(path)  # discards the warm-up records
    barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(traced):
        call()
    e.record()
    torch.cuda.synchronize()
    barrier()
    ms = torch.tensor([s.elapsed_time(e) / traced], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    comm.dump_trace(path)
    with open(path) as f:
        mine = summarise(json.load(f))
    os.unlink(path)
    everyone = [None] * world
    dist.all_gather_object(everyone, {"rank": rank, "launches": mine})
    if buffers == "registered" and world > 1:
        comm.deregister(x)
        comm.deregister(y)
    del x, y
    return {"op": op, "bytes_per_rank": n * es, "dtype": dtype, "ranks": world, "algo_requested": algo_name,
            "algo": comm.last_algorithm, "buffers": buffers,
            "event_us_per_call_max_over_ranks": round(float(ms.item()) * 1e3, 2),
            "traced_calls": traced, "ranks_detail": everyone}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--op", default="allreduce", choices=["allreduce", "broadcast", "reduce", "allgather",
                                                         "reducescatter"])
    p.add_argument("--bytes", default="128M", help="payload per rank (AllGather/ReduceScatter: per-rank block)")
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--algo", default="auto", choices=["auto", "oneshot", "twoshot", "nvls", "ring", "hybrid", "ll"])
    p.add_argument("--buffers", default="plain", choices=["plain", "registered", "symmetric"])
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--traced", type=int, default=3)
    p.add_argument("--records", type=int, default=1 << 20, help="trace buffer capacity (BCCL_TRACE)")
    p.add_argument("--cases", default="", help="comma list of op:bytes[:algo[:dtype[:buffers]]] (overrides the above)")
    p.add_argument("--out", default="", help="also append the summary records to this JSON-lines file")
    args = p.parse_args(argv)
    os.environ.setdefault("BCCL_TRACE", str(args.records))

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200.utils.results import ResultLog
    from originccl_b200.utils.sweep import parse_size

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731
    cases = []
    if args.cases:
        for spec in filter(None, (c.strip() for c in args.cases.split(","))):
            f = spec.split(":")
            f += [""] * (5 - len(f))
            cases.append((f[0], f[1], f[2] or "auto", f[3] or args.dtype, f[4] or args.buffers))
    else:
        cases.append((args.op, args.bytes, args.algo, args.dtype, args.buffers))
    log = ResultLog("trace_bench", args.out, enabled=rank == 0)
    for op, nbytes, algo_name, dtype, buffers in cases:
        rec = trace_case(comm, op, parse_size(nbytes), algo_name, dtype, buffers, args.warmup, args.traced, barrier)
        if rank == 0:
            log(json.dumps(rec))
    log.close()
    comm.destroy()
    barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
