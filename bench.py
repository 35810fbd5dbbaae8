"""Headline benchmark: AllReduce bus bandwidth on B200 (fp32, 128 MiB per rank).

One step = one out-of-place fp32 SUM AllReduce of ``--bytes`` per rank through this library's
device communicator. Launch with N=1 as ``python bench.py``; for N>1 under torchrun (one rank per
GPU). Rank 0 prints one JSON line:

* ``value``: NCCL bus bandwidth per rank (algbw * 2(N-1)/N, time = max over ranks), the
  convention the metric names; ``config.busbw_gbs_summed_over_ranks`` gives N times it. For N=1
  there is no bus (2(N-1)/N = 0): the single-rank AllReduce is a device copy and ``value`` is its
  algbw, flagged in ``config.n1_semantics``.
* ``ms_per_step``: device time per AllReduce (CUDA events, max over ranks).
* ``e2e``: the same metric through the public Python API with the step's input copied from
  pinned host memory and a sample of the result read back every step.
* ``nccl``: the same op (out of place on the same rotating inputs, or in place with
  ``--inplace``) through NCCL called directly on the same box, for comparison.
* ``zero_copy_arms`` (N>1): the same out-of-place op timed again on the same tensors registered
  with the communicator (``register``: peer memory, no staging copies; the default arm) and,
  with ``--zero-copy-arms registered,symmetric``, on symmetric multicast-bound allocations
  (``symmetric_empty``), each with its algorithm and error against NCCL's reduction. The
  headline ``value`` stays on plain, unregistered tensors.

``--impl reference`` runs the reference's own code path; the reference is a CMake C++ project
without a Python package and cannot be built on this image, so that arm prints an
``unavailable`` line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Published busbw of the reference at 128 MiB, fp32 SUM, OCCL auto, 1 host x 4 ranks over shared
# memory (README.md:223): 7.52 GB/s per rank.
REFERENCE_BUSBW_GBS = 7.52

REFERENCE_UNAVAILABLE = (
    "reference (qichen1336/OriginCCL) is a CPU-only CMake C++17 library with no setup.py/pyproject "
    "(pip install fails: 'not installable') and a hard dependency on libibverbs/librdmacm/fmt/MPI, "
    "none of which exist on this image; it has no GPU code path to run")


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--bytes", type=int, default=128 << 20, help="payload per rank")
    p.add_argument("--dtype", default="float32", choices=["float32", "bfloat16"])
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-nccl", action="store_true", help="skip the NCCL comparison")
    p.add_argument("--inplace", action="store_true", help="in-place AllReduce (default: out of place)")
    p.add_argument("--algo", default="auto", choices=["auto", "oneshot", "twoshot", "nvls", "ring", "hybrid", "ll"],
                   help="force one algorithm (default: the planner's choice)")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--no-clocks", action="store_true", help="diagnostic: do not sample clocks (no clocks key)")
    p.add_argument("--buffers", default="plain", choices=["plain", "registered", "symmetric"],
                   help="plain torch tensors (default); the same tensors registered with the communicator "
                        "(zero-copy over peer memory); or symmetric multicast-bound allocations (zero-copy NVLS)")
    p.add_argument("--zero-copy-arms", default="registered",
                   help="N>1, plain headline: comma list of extra arms that time the same op on other buffers "
                        "('registered': the same tensors registered with the communicator; 'symmetric': "
                        "multicast-bound allocations); 'none' to skip")
    return p.parse_args()


def main() -> None:
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}), flush=True)
        return
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    import torch
    import torch.distributed as dist

    import originccl_b200 as occl
    from originccl_b200.utils.clocks import ClockSampler
    from originccl_b200.utils.timing import busbw_factor

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
        comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
        barrier = lambda: dist.barrier(device_ids=[local])  # noqa: E731
    else:
        comm = occl.Communicator().init(0, 1, None, device=0)
        barrier = lambda: None  # noqa: E731

    dtype = {"float32": torch.float32, "bfloat16": torch.bfloat16}[args.dtype]
    esize = torch.empty((), dtype=dtype).element_size()
    count = args.bytes // esize
    nbytes = count * esize
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    # Two rotating inputs + output: 3 x 128 MiB on every rank, larger than the 126 MB L2.
    xs = [(torch.rand(count, device="cuda", generator=g) * 2 - 1).to(dtype) for _ in range(2)]
    y = torch.empty(count, device="cuda", dtype=dtype)
    if args.buffers == "symmetric" and world > 1:
        sym = [comm.symmetric_empty((count,), dtype) for _ in range(3)]
        for dst, src in zip(sym, xs):
            dst.copy_(src)
        torch.cuda.synchronize()
        xs, y = sym[:2], sym[2]
    elif args.buffers == "registered" and world > 1:
        for t_ in (*xs, y):
            comm.register(t_)

    algo = getattr(occl.Algo, args.algo.upper())

    def step(i: int) -> None:
        if args.inplace:
            comm.all_reduce(xs[i & 1], algo=algo)
        else:
            comm.all_reduce(xs[i & 1], out=y, algo=algo)

    def reference_of(i: int):
        """NCCL's fp32 AllReduce of step i's input (in-place steps change their input: only the
        first step of each buffer is checked then)."""
        ref = xs[i & 1].clone().float()
        if world > 1:
            dist.all_reduce(ref)
        return ref

    inputs0 = [x.clone() for x in xs] if args.inplace else None
    check = reference_of(0) if args.warmup > 0 else None
    for i in range(args.warmup):
        step(i)
        if i == 0 and check is not None:
            torch.cuda.synchronize()
            got = xs[0] if args.inplace else y
            max_err = float((got.float() - check).abs().max().item())
    torch.cuda.synchronize()
    if args.inplace:  # restore the inputs the warm-up reduced in place
        for x, x0 in zip(xs, inputs0):
            x.copy_(x0)
        del inputs0
    if args.warmup == 0:
        max_err = 0.0

    # Clocks of rank 0's GPU (NVML index = its position in CUDA_VISIBLE_DEVICES, if set).
    visible = [int(d) for d in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if d.strip().isdigit()]
    gpus = [visible[local] if local < len(visible) else local]
    launches0 = comm.kernel_launches
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        step(i)
    end.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = comm.kernel_launches - launches0
    algorithm = comm.last_algorithm
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())

    # The last timed step's output against NCCL's reduction of its input (out of place only:
    # in-place steps feed each output into a later step).
    last_err = None
    if not args.inplace:
        last_err = float((y.float() - reference_of(args.steps - 1)).abs().max().item())

    algbw = nbytes / (ms * 1e-3) / 1e9
    factor = busbw_factor("allreduce", world)
    busbw = algbw * factor
    value = busbw if world > 1 else algbw

    # NCCL on the same buffers and the same op (out of place on the rotating inputs, or in
    # place), called directly, with the same timing rules.
    nccl = None
    if world > 1 and not args.no_nccl:
        from originccl_b200.utils.nccl_direct import NcclDirect
        ncomm = NcclDirect(dist.distributed_c10d._get_default_store(), rank, world, local, tag="bench")
        saved = [x.clone() for x in xs] if args.inplace else None

        def nstep(i: int) -> None:
            if args.inplace:
                ncomm.all_reduce(xs[i & 1], xs[i & 1])
            else:
                ncomm.all_reduce(xs[i & 1], y)

        for i in range(args.warmup):
            nstep(i)
        torch.cuda.synchronize()
        barrier(); torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for i in range(args.steps):
            nstep(i)
        e2.record(); torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
        tn = torch.tensor([s2.elapsed_time(e2) / args.steps], dtype=torch.float64, device="cuda")
        dist.all_reduce(tn, op=dist.ReduceOp.MAX)
        nms = float(tn.item())
        nbus = nbytes / (nms * 1e-3) / 1e9 * factor
        nccl = {"ms_per_step": round(nms, 4), "busbw_gbs_per_rank": round(nbus, 2),
                "api": "ncclAllReduce (direct)", "inplace": args.inplace}
        if saved is not None:
            for x, x0 in zip(xs, saved):
                x.copy_(x0)
            del saved
        torch.cuda.synchronize()
        ncomm.destroy()

    # End to end through the public API: pinned H2D of this step's input, the collective, and a
    # device->host read of a 64 KiB sample of the result, every step (wall clock, max over ranks).
    host_in = [xs[i].cpu().pin_memory() for i in range(2)]
    dev_in = torch.empty_like(xs[0])
    sample = torch.empty(65536 // esize, dtype=dtype).pin_memory()
    for i in range(2):
        dev_in.copy_(host_in[i], non_blocking=True); comm.all_reduce(dev_in, out=y)
        sample.copy_(y[: sample.numel()], non_blocking=True); torch.cuda.synchronize()
    barrier(); torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        dev_in.copy_(host_in[i & 1], non_blocking=True)
        comm.all_reduce(dev_in, out=y)
        sample.copy_(y[: sample.numel()], non_blocking=True)
        torch.cuda.synchronize()
        _ = float(sample[0])
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    te = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item())
    e2e_algbw = nbytes / (e2e_ms * 1e-3) / 1e9
    e2e_value = e2e_algbw * factor if world > 1 else e2e_algbw

    # Clocks and throttle reasons under the same load: the same AllReduce loop for ~200 ms after
    # the measurements, sampled through NVML on rank 0's GPU. NVML queries during the timed loop
    # itself (even one sample before it) slowed the 2-GPU loop 1.9x (0.535 vs 0.282 ms per step),
    # so no measured loop runs with them; clock locks and throttling persist far longer than
    # this window, so it shows the state the timed region ran in.
    n_clk = max(20, int(200.0 / max(ms, 1e-3)))
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpus if rank == 0 and not args.no_clocks else [], interval_ms=10.0) as clocks:
        for i in range(n_clk):
            step(i)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    # Zero-copy arms (N>1, plain headline only): the same out-of-place AllReduce, same sizes and
    # timing rules, first on the same torch tensors registered with the communicator (peer
    # memory, no staging), then on symmetric multicast-bound allocations (NVLS without staging
    # where the planner picks NVLS). Reported beside the headline, which stays on plain buffers.
    def zero_copy_arm(kind: str) -> dict:
        """The same out-of-place AllReduce on registered tensors or symmetric allocations."""
        if kind == "registered":
            bufs = [*xs, y]
            for t_ in bufs:
                comm.register(t_)
        else:
            bufs = [comm.symmetric_empty((count,), dtype) for _ in range(3)]
            for dst_, src_ in zip(bufs[:2], xs):
                dst_.copy_(src_)
            torch.cuda.synchronize()
        zin, zout = bufs[:2], bufs[2]
        try:
            for i in range(args.warmup):
                comm.all_reduce(zin[i & 1], out=zout, algo=algo)
            torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
            s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0 = comm.kernel_launches
            s3.record()
            for i in range(args.steps):
                comm.all_reduce(zin[i & 1], out=zout, algo=algo)
            e3.record(); torch.cuda.synchronize(); barrier(); torch.cuda.synchronize()
            tz = torch.tensor([s3.elapsed_time(e3) / args.steps], dtype=torch.float64, device="cuda")
            dist.all_reduce(tz, op=dist.ReduceOp.MAX)
            zms = float(tz.item())
            zerr = float((zout.float() - ref_last).abs().max().item())
            return {"ms_per_step": round(zms, 4),
                    "busbw_gbs_per_rank": round(nbytes / (zms * 1e-3) / 1e9 * factor, 2),
                    "algorithm": comm.last_algorithm, "gpu_launches": comm.kernel_launches - l0,
                    "max_abs_err_vs_nccl_last_step": zerr}
        finally:
            if kind == "registered":
                for t_ in bufs:
                    comm.deregister(t_)
            torch.cuda.synchronize(); barrier()

    zero_copy = None
    arms = [a for a in args.zero_copy_arms.split(",") if a in ("registered", "symmetric")]
    if world > 1 and args.buffers == "plain" and arms and not args.inplace:
        zero_copy = {}
        ref_last = reference_of(args.steps - 1)
        for kind in arms:
            try:
                zero_copy[kind] = zero_copy_arm(kind)
            except Exception as e:  # noqa: BLE001  an extra arm must not cost the headline line
                # A failing library call fails the same way on every rank (registration and the
                # kernels' bounded waits are collective), so the ranks stay in step.
                zero_copy[kind] = {"error": f"{type(e).__name__}: {e}"[:300]}
                break
    if rank == 0:
        out = {
            "metric": "AllReduce bus GB/s vs size at 2/4/8 B200 (max over ranks) vs reference & NCCL",
            "value": round(value, 2),
            "unit": "GB/s (bus bandwidth per rank)" if world > 1 else "GB/s (algbw of a one-rank copy)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(value / REFERENCE_BUSBW_GBS, 2),
            "dtype": {"float32": "fp32", "bfloat16": "bf16"}[args.dtype],
            "buffers": args.buffers,
            "data": "synthetic (uniform [-1,1), seed 1234+rank)",
            "config": {
                "model": f"AllReduce SUM {'in-place' if args.inplace else 'out-of-place'}, {args.dtype}",
                "global_batch": world,
                "seq_len": count,
                "parallelism": f"dp{world}",
                "bytes_per_rank": nbytes,
                "busbw_gbs_per_rank": round(busbw, 2),
                "busbw_gbs_summed_over_ranks": round(busbw * world, 2),
                "inplace": args.inplace,
                "algbw_gbs": round(algbw, 2),
                "algorithm": algorithm,
                "buffers": args.buffers,
                "nvls": comm.nvls_enabled,
                "l2": "inputs larger than L2: two rotating 128 MiB inputs + a 128 MiB output per rank",
                "n1_semantics": ("N=1 has no bus (factor 2(N-1)/N = 0); value is the algbw of the single-rank "
                                 "AllReduce (a device copy)") if world == 1 else None,
                "max_abs_err_vs_nccl": {"first_warmup_step": max_err, "last_timed_step": last_err},
                "baseline_number": "reference 7.52 GB/s busbw per rank, 4 ranks, 128 MiB fp32 (README.md:223)",
            },
            "nccl": nccl,
            "zero_copy_arms": zero_copy,
            "e2e": {"value": round(e2e_value, 2),
                    "unit": "GB/s (bus bandwidth per rank)" if world > 1 else "GB/s (algbw of a one-rank copy)",
                    "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": nbytes,
                    "d2h_bytes_per_step": sample.numel() * esize, "steps": args.e2e_steps,
                    "api": "originccl_b200.Communicator.all_reduce"},
            "gpu_launches": launches,
            "clocks": {**clocks.summary(), "window": f"{n_clk} more steps of the same loop after the timed, "
                        "NCCL and e2e loops (NVML during a timed loop perturbs it)"},
        }
        print(json.dumps(out), flush=True)
    try:
        comm.destroy()
    except Exception as e:  # noqa: BLE001  after a failed extra arm; the line is out already
        print(f"rank {rank}: communicator teardown: {e}", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
