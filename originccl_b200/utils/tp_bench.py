"""Tensor-parallel Llama-style MLP benchmark: fused kernels vs NCCL + cuBLAS.

``torchrun --nproc-per-node 8 -m originccl_b200.utils.tp_bench`` runs X [tokens, hidden] sequence-
sharded over the ranks through AllGather->GEMM(SiLU) and GEMM->ReduceScatter, random-init
normal(0, 0.02) weights, bf16. Timing: CUDA events, warm-up, max over ranks. Reports ms per MLP
forward, TFLOP/s per GPU, and the fraction of the roofline max(FLOPs / measured GEMM peak,
NVLink bytes / 770 GB/s).
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys


def measured_peak_tflops(default: float = 1383.8) -> float:
    """The sustained cuBLAS bf16 peak measured on this pool's B200s (``bf16_tflops_sustained`` in
    the repository's MEASURED_PEAKS.json, written per machine pool), else ``default`` (an earlier
    measurement of the same loop)."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        import json
        with open(path) as f:
            return float(json.load(f)["bf16_tflops_sustained"])
    except (OSError, ValueError, KeyError, TypeError):
        return default


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--hidden", type=int, default=8192)
    p.add_argument("--ffn", type=int, default=28672)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--gemm-peak-tflops", type=float, default=None,
                   help="sustained bf16 GEMM peak for the roofline (default: MEASURED_PEAKS.json, else 1383.8)")
    p.add_argument("--nvlink-gbs", type=float, default=770.0)
    p.add_argument("--out", default="", help="also append the record to this JSON-lines file")
    p.add_argument("--variants", default="",
                   help="also time the fused MLP under each environment variant, e.g. "
                        "'BCCL_GEMM_BN=auto,BCCL_TP_PUSH_WARPS=2,BCCL_GEMM_BN=auto;BCCL_TP_PUSH_WARPS=2'")
    args = p.parse_args(argv)
    if args.gemm_peak_tflops is None:
        args.gemm_peak_tflops = measured_peak_tflops()
    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200.parallel.tensor_parallel import TensorParallelMLP

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
        comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local)
    else:
        comm = occl.Communicator().init(0, 1, None, device=0)
    mlp = TensorParallelMLP(comm, args.hidden, args.ffn, seed=3)
    ms = args.tokens // world
    g = torch.Generator(device="cuda").manual_seed(42 + rank)
    x = (torch.randn(ms, args.hidden, device="cuda", generator=g)).bfloat16()

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ours = timed(lambda: mlp(x))
    ref = timed(lambda: mlp.forward_reference(x))
    y = mlp(x)
    yr = mlp.forward_reference(x)
    torch.cuda.synchronize()
    rel = ((y.float() - yr.float()).abs().max() / yr.float().abs().max()).item()
    flops = 2 * 2.0 * args.tokens * args.hidden * (args.ffn // world)  # per rank, both GEMMs
    nvlink_bytes = 2 * (world - 1) * ms * args.hidden * 2  # AG in + RS out per rank, bf16
    roof_ms = max(flops / (args.gemm_peak_tflops * 1e12), nvlink_bytes / (args.nvlink_gbs * 1e9)) * 1e3
    # Where the time goes: each fused op alone, the same GEMMs without communication (this
    # library's kernel and cuBLAS) and the NCCL collectives alone.
    from originccl_b200.ops import gemm as gemm_op
    from originccl_b200.ops import tp as tp_op
    xg = torch.empty(args.tokens, args.hidden, device="cuda", dtype=torch.bfloat16)
    h = tp_op.all_gather_gemm(comm, x, mlp.w_up, "silu")
    part = torch.empty(args.tokens, args.hidden, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(ms, args.hidden, device="cuda", dtype=torch.bfloat16)
    bd = {
        "ag_gemm_ms": timed(lambda: tp_op.all_gather_gemm(comm, x, mlp.w_up, "silu", out=h)),
        "gemm_rs_ms": timed(lambda: tp_op.gemm_reduce_scatter(comm, h, mlp.w_down, out=out)),
        "gemm_up_ours_ms": timed(lambda: gemm_op.gemm(xg, mlp.w_up, "silu", out=h)),
        "gemm_down_ours_ms": timed(lambda: gemm_op.gemm(h, mlp.w_down, out=part)),
        "gemm_up_cublas_ms": timed(lambda: torch.matmul(xg, mlp.w_up.t())),
        "gemm_down_cublas_ms": timed(lambda: torch.matmul(h, mlp.w_down.t())),
    }
    if world > 1:
        bd["nccl_allgather_ms"] = timed(lambda: dist.all_gather_into_tensor(xg, x))
        bd["nccl_reducescatter_ms"] = timed(lambda: dist.reduce_scatter_tensor(out, part))
    bd = {k: round(v, 4) for k, v in bd.items()}
    # Knob variants (read by the kernels' launchers at every call, so they apply in-process).
    variants = {}
    for spec in filter(None, args.variants.split(",")):
        saved = {}
        for kv in spec.split(";"):
            k, _, v = kv.partition("=")
            saved[k] = os.environ.get(k)
            os.environ[k] = v
        variants[spec] = round(timed(lambda: mlp(x)), 4)
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    from originccl_b200.utils.results import ResultLog
    with ResultLog("tp_bench", args.out, enabled=rank == 0) as log:
        log({"bench": "tp_mlp", "world": world, "tokens": args.tokens, "hidden": args.hidden,
             "ffn": args.ffn, "ours_ms": round(ours, 4), "nccl_cublas_ms": round(ref, 4),
             "speedup": round(ref / ours, 3), "tflops_per_gpu": round(flops / ours / 1e9, 1),
             "roofline_ms": round(roof_ms, 4), "fraction_of_roofline": round(roof_ms / ours, 3),
             "gemm_peak_tflops": args.gemm_peak_tflops, "nvlink_gbs": args.nvlink_gbs,
             "max_rel_diff_vs_reference": rel, "gemm_kernel": gemm_op.kernel_name(args.tokens, args.ffn // world),
             "breakdown": bd, "variants_ms": variants})
    comm.destroy()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
