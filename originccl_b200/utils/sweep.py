"""Size sweep of one collective: this library vs NCCL (torch.distributed) on the same GPUs.

Run one rank per GPU::

    torchrun --nproc-per-node 8 -m originccl_b200.utils.sweep --op allreduce --dtype float32 \
        --min-bytes 8 --max-bytes 1G --out sweep.jsonl

Parity: the reference's AllReduce benchmark (OriginCCL tests/benchmark/test_allreduce_benchmark.cpp:
113-421) sweeps sizes by a factor, validates, and reports busbw = algbw * 2(N-1)/N with the time
taken as the max over ranks. Here every size is timed on the device with CUDA events (warm-up,
then ``iters`` calls between barriers + synchronize), the max over ranks is reported, and the
same buffers are timed through NCCL for comparison. Before timing, every size is checked once
against an fp64 reduction of the same inputs (``check`` in the record). Inputs are uniform in
[-1, 1] from seed 1234+rank. Rank 0 prints one JSON line per size. ``--graph K`` times CUDA-graph
replays of K captured calls instead of eager calls (both libraries), which removes the host's
launch path from small-message latency.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys


def parse_size(s: str) -> int:
    s = s.strip().upper()
    mult = 1
    for suf, m in (("K", 1 << 10), ("M", 1 << 20), ("G", 1 << 30)):
        if s.endswith(suf):
            mult, s = m, s[:-1]
    return int(float(s) * mult)


def run_sweep(comm, *, op: str, dtype: str, min_bytes: int, max_bytes: int, factor: int = 2, warmup: int = 20,
              iters: int = 100, algo: str = "auto", inplace: bool = False, nccl: bool = True, redop: str = "sum",
              seed: int = 1234, emit=print, graph: int = 0, buffers: str = "plain", ref_comm=None,
              variant: str = "") -> list:
    """Times ``op`` at every size from min_bytes to max_bytes (x factor) with this library and
    with NCCL on the same buffers; returns (and emits on rank 0) one record per size.

    ``graph`` > 0 captures that many back-to-back calls into one CUDA graph (for both
    libraries) and times graph replays instead of eager calls: the per-call time then excludes
    the host's launch path, as nccl-tests' ``-G`` does. ``buffers`` = ``"registered"`` registers
    this library's buffers with the communicator (zero-copy over peer memory) and
    ``"symmetric"`` allocates them in symmetric memory (zero-copy NVLS); NCCL uses plain copies
    of them. ``ref_comm`` (a ``utils.nccl_direct.NcclDirect``) times NCCL on exactly the same
    operation, out of place or in place like this library's; without it the NCCL arm goes through
    torch.distributed, whose collectives are in place."""
    import torch
    import torch.distributed as dist
    from originccl_b200 import Algo, ReduceOp
    from originccl_b200.utils.timing import busbw_factor

    rank, world, local = comm.rank, comm.world_size, comm.device
    dt = getattr(torch, dtype)
    es = torch.empty((), dtype=dt).element_size()
    algo_v = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS,
              "ring": Algo.RING, "hybrid": Algo.HYBRID, "ll": Algo.LL}[algo]
    rop = {"sum": ReduceOp.SUM, "max": ReduceOp.MAX, "min": ReduceOp.MIN, "avg": ReduceOp.AVG}[redop]
    nccl_op = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
               "avg": dist.ReduceOp.AVG}[redop]
    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731

    def timed(fn) -> float:
        if graph > 0:
            from originccl_b200.utils.graphs import capture, time_replays
            g = capture(fn, repeat=graph, warmup=warmup)
            g.replay()  # one untimed replay
            us = time_replays(g, max(1, iters // graph), graph, sync=barrier)
            t = torch.tensor([us], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            del g
            return float(t.item())
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / iters], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) * 1e3  # microseconds

    out = []
    size = max(min_bytes, es)
    g = torch.Generator(device="cuda").manual_seed(seed + rank)
    sym = [None, None]  # symmetric buffers (buffers="symmetric"), allocated on first use
    while size <= max_bytes:
        n = max(1, size // es)
        # Per-rank payload convention (as nccl-tests): allreduce/broadcast/reduce move n elements;
        # allgather gathers n per rank; reducescatter scatters n per rank (input world*n).
        if op == "reducescatter":
            x = (torch.rand(n * world, device="cuda", generator=g) * 2 - 1).to(dt)
            y = torch.empty(n, device="cuda", dtype=dt)
        elif op == "allgather":
            x = (torch.rand(n, device="cuda", generator=g) * 2 - 1).to(dt)
            y = torch.empty(n * world, device="cuda", dtype=dt)
        else:
            x = (torch.rand(n, device="cuda", generator=g) * 2 - 1).to(dt)
            y = x if inplace else torch.empty_like(x)
        registered = []
        if buffers == "symmetric" and world > 1:
            # Views at the start of two symmetric buffers sized once for the largest point (every
            # rank uses the same offsets, as the zero-copy kernels require).
            if sym[0] is None:
                cap = max(1, max_bytes // es) * world
                sym[0], sym[1] = comm.symmetric_empty((cap,), dt), comm.symmetric_empty((cap,), dt)
            xs_, ys_ = sym[0][:x.numel()], sym[1][:y.numel()]
            xs_.copy_(x)
            torch.cuda.synchronize()
            x, y = xs_, (xs_ if inplace and op not in ("reducescatter", "allgather") else ys_)
        elif buffers == "registered" and world > 1:
            for t_ in ({id(x): x, id(y): y}).values():
                comm.register(t_)
                registered.append(t_)
        rc = ref_comm
        if op == "allreduce":
            ours = lambda: comm.all_reduce(x, rop, out=y, algo=algo_v)  # noqa: E731
            ref = ((lambda: rc.all_reduce(x, y, redop)) if rc is not None  # noqa: E731
                   else (lambda: dist.all_reduce(y, op=nccl_op)))
            nbytes = n * es
        elif op == "allgather":
            ours = lambda: comm.all_gather(y, x)  # noqa: E731
            ref = ((lambda: rc.all_gather(x, y)) if rc is not None  # noqa: E731
                   else (lambda: dist.all_gather_into_tensor(y, x)))
            nbytes = n * es * world
        elif op == "reducescatter":
            ours = lambda: comm.reduce_scatter(y, x, rop)  # noqa: E731
            ref = ((lambda: rc.reduce_scatter(x, y, redop)) if rc is not None  # noqa: E731
                   else (lambda: dist.reduce_scatter_tensor(y, x, op=nccl_op)))
            nbytes = n * es * world
        elif op == "broadcast":
            ours = lambda: comm.broadcast(y, 0, src=x if rank == 0 else None, algo=algo_v)  # noqa: E731
            ref = ((lambda: rc.broadcast(x, y, 0)) if rc is not None  # noqa: E731
                   else (lambda: dist.broadcast(y, 0)))
            nbytes = n * es
        else:
            ours = lambda: comm.reduce(x, 0, rop, out=y, algo=algo_v)  # noqa: E731
            ref = ((lambda: rc.reduce(x, y, 0, redop)) if rc is not None  # noqa: E731
                   else (lambda: dist.reduce(y, 0, op=nccl_op)))
            nbytes = n * es
        ok = _check(comm, op, x, rop, nccl_op, dtype)
        t_ours = timed(ours)
        used = comm.last_algorithm
        t_nccl = timed(ref) if nccl else None
        f = busbw_factor(op, world)
        rec = {"op": op, "dtype": dtype, "redop": redop, "bytes": n * es, "ranks": world, "algo": used,
               "time_us": round(t_ours, 3), "algbw_gbs": round(nbytes / t_ours / 1e3, 3),
               "busbw_gbs": round(nbytes / t_ours / 1e3 * f, 3), "inplace": inplace, "check": ok,
               "graph": graph, "buffers": buffers, "nccl_api": "direct" if rc is not None else "torch.distributed"}
        if variant:
            rec["variant"] = variant
        if t_nccl is not None:
            rec.update({"nccl_time_us": round(t_nccl, 3), "nccl_busbw_gbs": round(nbytes / t_nccl / 1e3 * f, 3),
                        "speedup_vs_nccl": round(t_nccl / t_ours, 3)})
        if rank == 0:
            emit(json.dumps(rec))
        out.append(rec)
        for t_ in registered:
            comm.deregister(t_)
        del x, y
        size *= factor
    return out


_RTOL = {"float32": 1e-5, "bfloat16": 8e-3, "float16": 1e-3, "int32": 0.0}


def _check(comm, op: str, x, rop, nccl_op, dtype: str) -> bool:
    """One out-of-place call of ``op`` on ``x`` against an fp64 NCCL reduction of the same inputs
    (exact comparison for the data-movement ops); the verdict is agreed over all ranks."""
    import torch
    import torch.distributed as dist
    rank, world = comm.rank, comm.world_size
    n = x.numel()
    x64 = x.double() if dtype != "int32" else x.long()
    if op == "allreduce":
        got = torch.empty_like(x)
        comm.all_reduce(x, rop, out=got)
        ref = x64.clone()
        dist.all_reduce(ref, op=nccl_op)
    elif op == "reducescatter":
        m = n // world
        got = torch.empty(m, dtype=x.dtype, device=x.device)
        comm.reduce_scatter(got, x, rop)
        ref = x64.clone()
        dist.all_reduce(ref, op=nccl_op)
        ref = ref[rank * m:(rank + 1) * m]
    elif op == "reduce":
        got = torch.empty_like(x)
        comm.reduce(x, 0, rop, out=got)
        ref = x64.clone()
        dist.all_reduce(ref, op=nccl_op)
        if rank != 0:  # only the root's output is defined
            got = ref.to(x.dtype)
    elif op == "allgather":
        got = torch.empty(n * world, dtype=x.dtype, device=x.device)
        comm.all_gather(got, x)
        ref = torch.empty_like(got)
        dist.all_gather_into_tensor(ref, x)
    else:  # broadcast from root 0
        got = torch.empty_like(x)
        comm.broadcast(got, 0, src=x if rank == 0 else None)
        ref = x.clone()
        dist.broadcast(ref, 0)
    rtol = _RTOL[dtype]
    err = (got.double() - ref.double()).abs()
    bound = rtol * (ref.double().abs() + world)
    ok = torch.tensor([1 if bool((err <= bound).all()) else 0], device=x.device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    return bool(ok.item())


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--op", default="allreduce",
                   choices=["allreduce", "allgather", "reducescatter", "broadcast", "reduce"])
    p.add_argument("--dtype", default="float32",
                   help="comma list of float32, bfloat16, float16, int32 (each swept in turn)")
    p.add_argument("--redop", default="sum", choices=["sum", "max", "min", "avg"])
    p.add_argument("--min-bytes", default="8")
    p.add_argument("--max-bytes", default="1G")
    p.add_argument("--factor", type=int, default=2)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--iters", type=int, default=100)
    p.add_argument("--algo", default="auto",
                   help="comma list of auto, oneshot, twoshot, nvls, ring, hybrid, ll (each swept in turn)")
    p.add_argument("--variants", default="",
                   help="';'-separated environment variants, each a ','-separated list of NAME=VALUE set "
                        "while a fresh communicator initialises (e.g. 'BCCL_PIPE_LAG=2;BCCL_PIPE_LAG=1'); "
                        "every algorithm is swept under every variant")
    p.add_argument("--inplace", action="store_true")
    p.add_argument("--both-places", action="store_true", help="sweep out of place, then in place")
    p.add_argument("--no-nccl", action="store_true")
    p.add_argument("--out", default="", help="also append the records to this JSON-lines file")
    p.add_argument("--buffers", default="plain", choices=["plain", "registered", "symmetric"],
                   help="this library's buffers: plain tensors, registered tensors or symmetric memory")
    p.add_argument("--nccl-api", default="direct", choices=["direct", "torch"],
                   help="NCCL arm: ncclAllReduce & co. called directly on the same op (default) or "
                        "torch.distributed (in place)")
    p.add_argument("--graph", type=int, default=0,
                   help="capture this many calls per CUDA graph and time replays (0: eager calls)")
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    store = dist.distributed_c10d._get_default_store()
    from originccl_b200.utils.results import ResultLog
    log = ResultLog("sweep", args.out, enabled=rank == 0)

    ref_comm = None
    if not args.no_nccl and args.nccl_api == "direct":
        from originccl_b200.utils.nccl_direct import NcclDirect
        ref_comm = NcclDirect(store, rank, world, local, tag="sweep")
    dtypes = [d.strip() for d in args.dtype.split(",") if d.strip()]
    for d in dtypes:
        if d not in ("float32", "bfloat16", "float16", "int32"):
            raise SystemExit(f"unsupported dtype {d}")
    algos = [a.strip() for a in args.algo.split(",") if a.strip()]
    for a in algos:
        if a not in ("auto", "oneshot", "twoshot", "nvls", "ring", "hybrid", "ll"):
            raise SystemExit(f"unknown algorithm {a}")
    places = [False, True] if args.both_places else [args.inplace]
    variants = [v.strip() for v in args.variants.split(";")] if args.variants else [""]
    nccl_done = set()
    for variant in variants:
        saved = {}
        for kv in filter(None, (x.strip() for x in variant.split(","))):
            k, v = kv.split("=", 1)
            saved[k] = os.environ.get(k)
            os.environ[k] = v
        comm = occl.init_from_store(store, rank, world, device=local)
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        for d in dtypes:
            for inplace in places:
                for a in algos:
                    # NCCL once per (dtype, place): it does not depend on this library's settings.
                    want_nccl = not args.no_nccl and (d, inplace) not in nccl_done
                    nccl_done.add((d, inplace))
                    run_sweep(comm, op=args.op, dtype=d, min_bytes=parse_size(args.min_bytes),
                              max_bytes=parse_size(args.max_bytes), factor=args.factor, warmup=args.warmup,
                              iters=args.iters, algo=a, inplace=inplace, nccl=want_nccl, redop=args.redop,
                              emit=log, graph=args.graph, buffers=args.buffers, ref_comm=ref_comm, variant=variant)
        comm.destroy()
        dist.barrier(device_ids=[local])
    log.close()
    if ref_comm is not None:
        torch.cuda.synchronize()
        ref_comm.destroy()
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
