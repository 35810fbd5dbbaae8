"""Mixed collectives on one node: this library vs NCCL.

Run one rank per GPU::

    torchrun --nproc-per-node 8 -m originccl_b200.utils.mixed_bench

Parts (each timed with CUDA events, warm-up first, max over ranks; every result is checked):

* ``rs_ag``: ReduceScatter and AllGather, bf16, 1 KiB - 512 MiB per rank (``--max-bytes``);
* ``bcast_reduce``: Broadcast and Reduce (SUM and MAX), fp32, from root 0;
* ``sendrecv``: ring-neighbour Send/Recv of 4 MiB (every rank sends to rank+1 and receives from
  rank-1 in one group);
* ``group8``: batches of 8 independent operations (AllReduce SUM/MAX, AllGather, ReduceScatter,
  Broadcast, Reduce) issued inside nested GroupStart/GroupEnd, at ``--group-bytes`` per operation.
  This library runs a batch as one kernel; the NCCL arm issues the same 8 calls in order.

Values are normal(0, 1) from seed 42+rank. Rank 0 prints one JSON line per measurement.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--parts", default="rs_ag,bcast_reduce,sendrecv,group8")
    p.add_argument("--min-bytes", default="1K")
    p.add_argument("--max-bytes", default="512M")
    p.add_argument("--factor", type=int, default=4)
    p.add_argument("--group-bytes", default="4K,64K,1M")
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--iters", type=int, default=100)
    p.add_argument("--out", default="", help="also append the records to this JSON-lines file")
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200 import ReduceOp
    from originccl_b200.utils.sweep import parse_size, run_sweep

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731
    parts = set(args.parts.split(","))
    lo, hi = parse_size(args.min_bytes), parse_size(args.max_bytes)
    from originccl_b200.utils.results import ResultLog
    emit = ResultLog("mixed_bench", args.out, enabled=rank == 0)
    # The NCCL arm of the size sweeps calls ncclReduceScatter & co. directly on the same out-of-place
    # operation as this library (torch.distributed's broadcast / reduce work in place).
    from originccl_b200.utils.nccl_direct import NcclDirect
    ref_comm = NcclDirect(dist.distributed_c10d._get_default_store(), rank, world, local, tag="mixed")
    common = dict(factor=args.factor, warmup=args.warmup, iters=args.iters, seed=42, emit=emit, ref_comm=ref_comm)
    all_ok = True

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
        t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) * 1e3

    def agree(ok: bool) -> bool:
        t = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    if "rs_ag" in parts:
        for op in ("reducescatter", "allgather"):
            recs = run_sweep(comm, op=op, dtype="bfloat16", min_bytes=lo, max_bytes=hi, **common)
            all_ok &= all(r["check"] for r in recs)
    if "bcast_reduce" in parts:
        recs = run_sweep(comm, op="broadcast", dtype="float32", min_bytes=lo, max_bytes=hi, **common)
        for redop in ("sum", "max"):
            recs += run_sweep(comm, op="reduce", dtype="float32", min_bytes=lo, max_bytes=hi, redop=redop, **common)
        all_ok &= all(r["check"] for r in recs)

    g = torch.Generator(device=dev).manual_seed(42 + rank)
    if "sendrecv" in parts and world > 1:
        n = (4 << 20) // 4
        nxt, prv = (rank + 1) % world, (rank - 1) % world
        src = torch.randn(n, device=dev, generator=g)
        dst = torch.empty_like(src)

        def ours():
            with comm.group():
                comm.send(src, nxt)
                comm.recv(dst, prv)

        def nccl():
            ops = [dist.P2POp(dist.isend, src, nxt), dist.P2POp(dist.irecv, dst, prv)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()

        ours()
        torch.cuda.synchronize()
        expect = torch.empty_like(src)
        ops = [dist.P2POp(dist.isend, src, nxt), dist.P2POp(dist.irecv, expect, prv)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        ok = agree(torch.equal(dst, expect))
        all_ok &= ok
        t_o, t_n = timed(ours), timed(nccl)
        if rank == 0:
            emit(json.dumps({"op": "sendrecv_ring", "bytes": n * 4, "ranks": world, "time_us": round(t_o, 2),
                             "algbw_gbs": round(n * 4 / t_o / 1e3, 2), "nccl_time_us": round(t_n, 2),
                             "nccl_algbw_gbs": round(n * 4 / t_n / 1e3, 2), "speedup_vs_nccl": round(t_n / t_o, 3),
                             "check": ok, "transport": comm.p2p_transport(nxt)}))

    if "group8" in parts:
        for gb in args.group_bytes.split(","):
            nbytes = parse_size(gb)
            n = max(world, nbytes // 4) // world * world
            xs = [torch.randn(n, device=dev, generator=g) for _ in range(8)]
            outs = [torch.empty(n, device=dev) for _ in range(4)] + [torch.empty(n * world, device=dev),
                                                                      torch.empty(n // world, device=dev),
                                                                      torch.empty(n, device=dev),
                                                                      torch.empty(n, device=dev)]

            def ours():
                comm.group_start()
                comm.group_start()  # nested: only the outer group_end runs the batch
                comm.all_reduce(xs[0], ReduceOp.SUM, out=outs[0])
                comm.all_reduce(xs[1], ReduceOp.MAX, out=outs[1])
                comm.all_reduce(xs[2], ReduceOp.SUM, out=outs[2], scale=1.0 / world)
                comm.all_reduce(xs[3], ReduceOp.MIN, out=outs[3])
                comm.group_end()
                comm.all_gather(outs[4], xs[4])
                comm.reduce_scatter(outs[5], xs[5])
                comm.broadcast(outs[6], 0, src=xs[6] if rank == 0 else None)
                comm.reduce(xs[7], 0, ReduceOp.SUM, out=outs[7])
                comm.group_end()

            ref_outs = [torch.empty_like(o) for o in outs]

            def nccl(load_inputs: bool = False):
                # NCCL's AllReduce/Broadcast/Reduce work in place: inputs are copied in only for
                # the correctness pass, not in the timed calls.
                for i, o in zip(range(4), (dist.ReduceOp.SUM, dist.ReduceOp.MAX, dist.ReduceOp.AVG,
                                           dist.ReduceOp.MIN)):
                    if load_inputs:
                        ref_outs[i].copy_(xs[i])
                    dist.all_reduce(ref_outs[i], op=o)
                dist.all_gather_into_tensor(ref_outs[4], xs[4])
                dist.reduce_scatter_tensor(ref_outs[5], xs[5])
                if load_inputs and rank == 0:
                    ref_outs[6].copy_(xs[6])
                dist.broadcast(ref_outs[6], 0)
                if load_inputs:
                    ref_outs[7].copy_(xs[7])
                dist.reduce(ref_outs[7], 0)

            launches0 = comm.kernel_launches
            ours()
            torch.cuda.synchronize()
            launches = comm.kernel_launches - launches0
            nccl(load_inputs=True)
            torch.cuda.synchronize()
            ok = True
            for i, (a, b) in enumerate(zip(outs, ref_outs)):
                if i == 7 and rank != 0:
                    continue
                ok &= bool(torch.allclose(a, b, rtol=1e-5, atol=1e-5 * world))
            ok = agree(ok)
            all_ok &= ok
            t_o, t_n = timed(ours), timed(nccl)
            if rank == 0:
                emit(json.dumps({"op": "group8_nested", "bytes_per_op": n * 4, "ranks": world, "time_us": round(t_o, 2),
                                 "kernel_launches": launches, "nccl_time_us": round(t_n, 2),
                                 "speedup_vs_nccl": round(t_n / t_o, 3), "check": ok}))
            del xs, outs, ref_outs
    torch.cuda.synchronize()
    ref_comm.destroy()
    comm.destroy()
    barrier()
    dist.destroy_process_group()
    return 0 if all_ok else 1


if __name__ == "__main__":
    sys.exit(main())
