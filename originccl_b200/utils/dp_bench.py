"""Data-parallel gradient sync of an 8B-parameter Llama-3-shaped model: this library vs NCCL.

Run one rank per GPU::

    torchrun --nproc-per-node 8 -m originccl_b200.utils.dp_bench --steps 5 --warmup 3

Workload: every gradient of Llama-3-8B (8.03e9 bf16 values, 16 GB per rank)
in one flat buffer synced as 25 MiB buckets, each an AllReduce with the 1/world scale fused, plus
256 bias-style gradients of 4 KiB synced as one GroupStart/GroupEnd batch. Gradients are
normal(0, 1e-3) from seed 7+rank. The NCCL arm runs the same buckets with ``ReduceOp.AVG`` and the
256 small tensors inside one coalesced NCCL group. Each step is timed with CUDA events on the
launching stream (max over ranks); a step's 16 GB of buckets is far larger than L2, so no flush is
needed. Before timing, sampled buckets and the small tensors are checked against NCCL's result.
``--layers`` shrinks the model for quick runs (and is reported in the output).
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--bucket-mb", type=float, default=25.0)
    p.add_argument("--small", type=int, default=256, help="number of 4 KiB tensors in the group")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--no-nccl", action="store_true")
    p.add_argument("--out", default="", help="also append the record to this JSON-lines file")
    p.add_argument("--symmetric", action="store_true",
                   help="gradient buckets in the communicator's symmetric (multicast-bound) memory")
    p.add_argument("--register", action="store_true",
                   help="register the gradient storage with the communicator (zero-copy over peer memory)")
    p.add_argument("--also-register", action="store_true",
                   help="after the main measurement, time the same sync with the storage registered")
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200.models import LlamaConfig, param_shapes
    from originccl_b200.parallel.data_parallel import DataParallelSync, GradBuckets
    from originccl_b200.utils.timing import max_over_ranks

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731

    cfg = LlamaConfig(layers=args.layers)
    shapes = param_shapes(cfg) + [(f"bias.{i}", (2048,)) for i in range(args.small)]
    grads = GradBuckets(shapes, dtype=torch.bfloat16, device=dev, bucket_bytes=int(args.bucket_mb * (1 << 20)),
                        small_bytes=4096, allocator=comm.symmetric_empty if args.symmetric else None)
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    chunk = 1 << 28
    for lo in range(0, grads.flat.numel(), chunk):
        seg = grads.flat[lo:lo + chunk]
        seg.copy_(torch.randn(seg.numel(), device=dev, generator=gen) * 1e-3)
    grads.small_flat.copy_(torch.randn(grads.small_flat.numel(), device=dev, generator=gen) * 1e-3)
    dp = DataParallelSync(comm, grads, register=args.register)
    small = grads.small_tensors()
    nb = grads.num_buckets

    def nccl_step():
        for i in range(nb):
            dist.all_reduce(grads.bucket(i), op=dist.ReduceOp.AVG)
        with dist.distributed_c10d._coalescing_manager(device=dev):
            for t in small:
                dist.all_reduce(t, op=dist.ReduceOp.AVG)

    # Check: a few buckets and the small tensors, ours vs NCCL on identical copies.
    sample = sorted({0, nb // 2, nb - 1})
    before = [grads.bucket(i).clone() for i in sample]
    before_small = grads.small_flat.clone()
    dp.sync()
    ours_out = [grads.bucket(i).clone() for i in sample]
    ours_small = grads.small_flat.clone()
    for t in before:
        dist.all_reduce(t, op=dist.ReduceOp.AVG)
    dist.all_reduce(before_small, op=dist.ReduceOp.AVG)
    worst = 0.0
    for a, b in zip(ours_out + [ours_small], before + [before_small]):
        d = ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()
        worst = max(worst, d)
    ok = worst < 2e-2
    del before, before_small, ours_out, ours_small

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            fn()
        e.record()
        torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / args.steps)

    t_ours = timed(dp.sync)
    launches0 = comm.kernel_launches
    dp.sync()
    torch.cuda.synchronize()
    launches = comm.kernel_launches - launches0
    t_small = timed(lambda: dp._sync_small(torch.cuda.current_stream()))
    t_nccl = t_small_nccl = None
    if not args.no_nccl and world > 1:
        t_nccl = timed(nccl_step)

        def nccl_small():
            with dist.distributed_c10d._coalescing_manager(device=dev):
                for t in small:
                    dist.all_reduce(t, op=dist.ReduceOp.AVG)
        t_small_nccl = timed(nccl_small)
    from originccl_b200 import ReduceOp
    comm.all_reduce(grads.bucket(0), ReduceOp.SUM, scale=1.0 / world)  # untimed: which kernel a bucket uses
    bucket_algo = comm.last_algorithm
    reg = None
    if args.also_register and not args.register and world > 1:
        dp_reg = DataParallelSync(comm, grads, register=True)
        t_reg = timed(dp_reg.sync)
        comm.all_reduce(grads.bucket(0), ReduceOp.SUM, scale=1.0 / world)
        reg = {"registered_ms_per_sync": round(t_reg, 3), "registered_bucket_algorithm": comm.last_algorithm}
        dp_reg.close()
    nbytes = grads.numel * 2
    f = 2.0 * (world - 1) / world if world > 1 else 1.0
    rec = {"workload": "dp_grad_sync", "model": f"llama3-8b-shaped ({args.layers} layers)", "ranks": world,
           "symmetric_buckets": args.symmetric, "registered_buckets": args.register, "bucket_algorithm": bucket_algo,
           "grad_values": grads.numel, "bucket_mb": args.bucket_mb, "buckets": nb, "small_tensors": len(small),
           "ms_per_sync": round(t_ours, 3), "busbw_gbs": round(nbytes / t_ours / 1e6 * f, 1),
           "launches_per_sync": launches, "small_group_us": round(t_small * 1e3, 2), "check_rel_err": worst,
           "ok": ok, "steps": args.steps, "warmup": args.warmup}
    if reg is not None:
        rec.update(reg)
        if t_nccl is not None:
            rec["registered_speedup_vs_nccl"] = round(t_nccl / reg["registered_ms_per_sync"], 3)
    if t_nccl is not None:
        rec.update({"nccl_ms_per_sync": round(t_nccl, 3), "nccl_busbw_gbs": round(nbytes / t_nccl / 1e6 * f, 1),
                    "speedup_vs_nccl": round(t_nccl / t_ours, 3), "nccl_small_group_us": round(t_small_nccl * 1e3, 2)})
    from originccl_b200.utils.results import ResultLog
    with ResultLog("dp_bench", args.out, enabled=rank == 0) as log:
        log(rec)
    dp.close()
    comm.destroy()
    barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
