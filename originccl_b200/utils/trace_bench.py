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


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--op", default="allreduce", choices=["allreduce", "broadcast", "reduce", "allgather",
                                                         "reducescatter"])
    p.add_argument("--bytes", default="128M", help="payload per rank (AllGather/ReduceScatter: per-rank block)")
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--algo", default="auto", choices=["auto", "oneshot", "twoshot", "nvls", "ring", "hybrid"])
    p.add_argument("--buffers", default="plain", choices=["plain", "registered", "symmetric"])
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--traced", type=int, default=3)
    p.add_argument("--records", type=int, default=1 << 20, help="trace buffer capacity (BCCL_TRACE)")
    p.add_argument("--out", default="", help="also append the summary records to this JSON-lines file")
    args = p.parse_args(argv)
    os.environ.setdefault("BCCL_TRACE", str(args.records))

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200 import Algo
    from originccl_b200.utils.results import ResultLog
    from originccl_b200.utils.sweep import parse_size

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    dt = getattr(torch, args.dtype)
    es = torch.empty((), dtype=dt).element_size()
    n = max(1, parse_size(args.bytes) // es)
    algo = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS,
            "ring": Algo.RING, "hybrid": Algo.HYBRID}[args.algo]
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    nin = n * world if args.op == "reducescatter" else n
    nout = n * world if args.op == "allgather" else n
    alloc = (lambda m: comm.symmetric_empty((m,), dt)) if args.buffers == "symmetric" and world > 1 else \
        (lambda m: torch.empty(m, device="cuda", dtype=dt))
    x, y = alloc(nin), alloc(nout)
    x.copy_((torch.rand(nin, device="cuda", generator=g) * 2 - 1).to(dt))
    if args.buffers == "registered" and world > 1:
        comm.register(x)
        comm.register(y)

    def call() -> None:
        if args.op == "allreduce":
            comm.all_reduce(x, out=y, algo=algo)
        elif args.op == "broadcast":
            comm.broadcast(y, 0, src=x if rank == 0 else None, algo=algo)
        elif args.op == "reduce":
            comm.reduce(x, 0, out=y, algo=algo)
        elif args.op == "allgather":
            comm.all_gather(y, x, algo=algo)
        else:
            comm.reduce_scatter(y, x, algo=algo)

    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    path = os.path.join(tempfile.gettempdir(), f"bccl_trace_{os.getpid()}.json")
    comm.dump_trace(path)  # discards the warm-up records
    barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.traced):
        call()
    e.record()
    torch.cuda.synchronize()
    barrier()
    ms = torch.tensor([s.elapsed_time(e) / args.traced], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    comm.dump_trace(path)
    with open(path) as f:
        mine = summarise(json.load(f))
    os.unlink(path)
    everyone = [None] * world
    dist.all_gather_object(everyone, {"rank": rank, "launches": mine})
    if rank == 0:
        log = ResultLog("trace_bench", args.out, enabled=True)
        log(json.dumps({"op": args.op, "bytes_per_rank": n * es, "dtype": args.dtype, "ranks": world,
                        "algo": comm.last_algorithm, "buffers": args.buffers,
                        "event_us_per_call_max_over_ranks": round(float(ms.item()) * 1e3, 2),
                        "traced_calls": args.traced, "ranks_detail": everyone}))
        log.close()
    comm.destroy()
    barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
