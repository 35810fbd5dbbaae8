"""Size sweep of one collective: this library vs NCCL (torch.distributed) on the same GPUs.

Run one rank per GPU::

    torchrun --nproc-per-node 8 -m originccl_b200.utils.sweep --op allreduce --dtype float32 \
        --min-bytes 8 --max-bytes 1G --out sweep.jsonl

Parity: the reference's AllReduce benchmark (OriginCCL tests/benchmark/test_allreduce_benchmark.cpp:
113-421) sweeps sizes by a factor, validates, and reports busbw = algbw * 2(N-1)/N with the time
taken as the max over ranks. Here every size is timed on the device with CUDA events (warm-up,
then ``iters`` calls between barriers + synchronize), the max over ranks is reported, and the
same buffers are timed through NCCL for comparison. Rank 0 prints one JSON line per size.
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


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--op", default="allreduce",
                   choices=["allreduce", "allgather", "reducescatter", "broadcast", "reduce"])
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16", "float16", "int32"])
    p.add_argument("--min-bytes", default="8")
    p.add_argument("--max-bytes", default="1G")
    p.add_argument("--factor", type=int, default=2)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--iters", type=int, default=100)
    p.add_argument("--algo", default="auto", choices=["auto", "oneshot", "twoshot", "nvls"])
    p.add_argument("--inplace", action="store_true")
    p.add_argument("--no-nccl", action="store_true")
    p.add_argument("--out", default="")
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200 import Algo
    from originccl_b200.utils.timing import busbw_factor

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    dtype = getattr(torch, args.dtype)
    es = torch.empty((), dtype=dtype).element_size()
    algo = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS}[args.algo]
    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731

    def timed(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) * 1e3  # microseconds

    out_f = open(args.out, "a") if (args.out and rank == 0) else None
    size = max(parse_size(args.min_bytes), es)
    max_b = parse_size(args.max_bytes)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    while size <= max_b:
        n = max(1, size // es)
        # Per-rank payload convention (as nccl-tests): allreduce/broadcast/reduce move n elements;
        # allgather gathers n per rank; reducescatter scatters n per rank (input world*n).
        if args.op == "reducescatter":
            x = torch.rand(n * world, device="cuda", generator=g).to(dtype)
            y = torch.empty(n, device="cuda", dtype=dtype)
        elif args.op == "allgather":
            x = torch.rand(n, device="cuda", generator=g).to(dtype)
            y = torch.empty(n * world, device="cuda", dtype=dtype)
        else:
            x = torch.rand(n, device="cuda", generator=g).to(dtype)
            y = x if args.inplace else torch.empty_like(x)
        if args.op == "allreduce":
            ours = lambda: comm.all_reduce(x, out=y, algo=algo)  # noqa: E731
            ref = lambda: dist.all_reduce(y)  # noqa: E731
            nbytes = n * es
        elif args.op == "allgather":
            ours = lambda: comm.all_gather(y, x)  # noqa: E731
            ref = lambda: dist.all_gather_into_tensor(y, x)  # noqa: E731
            nbytes = n * es * world
        elif args.op == "reducescatter":
            ours = lambda: comm.reduce_scatter(y, x)  # noqa: E731
            ref = lambda: dist.reduce_scatter_tensor(y, x)  # noqa: E731
            nbytes = n * es * world
        elif args.op == "broadcast":
            ours = lambda: comm.broadcast(y, 0, src=x if rank == 0 else None, algo=algo)  # noqa: E731
            ref = lambda: dist.broadcast(y, 0)  # noqa: E731
            nbytes = n * es
        else:
            ours = lambda: comm.reduce(x, 0, out=y, algo=algo)  # noqa: E731
            ref = lambda: dist.reduce(y, 0)  # noqa: E731
            nbytes = n * es
        t_ours = timed(ours)
        used = comm.last_algorithm
        t_nccl = None if args.no_nccl else timed(ref)
        f = busbw_factor(args.op, world)
        rec = {"op": args.op, "dtype": args.dtype, "bytes": n * es, "ranks": world, "algo": used,
               "time_us": round(t_ours, 3), "algbw_gbs": round(nbytes / t_ours / 1e3, 3),
               "busbw_gbs": round(nbytes / t_ours / 1e3 * f, 3), "inplace": args.inplace}
        if t_nccl is not None:
            rec.update({"nccl_time_us": round(t_nccl, 3), "nccl_busbw_gbs": round(nbytes / t_nccl / 1e3 * f, 3),
                        "speedup_vs_nccl": round(t_nccl / t_ours, 3)})
        if rank == 0:
            line = json.dumps(rec)
            print(line, flush=True)
            if out_f:
                out_f.write(line + "\n")
                out_f.flush()
        del x, y
        size *= args.factor
    if out_f:
        out_f.close()
    comm.destroy()
    barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
