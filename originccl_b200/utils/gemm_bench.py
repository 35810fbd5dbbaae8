"""tcgen05 bf16 GEMM against cuBLAS (``torch.matmul``) on the tensor-parallel MLP shapes.

    python -m originccl_b200.utils.gemm_bench                 # default kernel choice
    BCCL_GEMM_PAIR=1 python -m originccl_b200.utils.gemm_bench   # force the 2-SM kernel
    BCCL_GEMM_PAIR=0 python -m originccl_b200.utils.gemm_bench   # force the 1-SM kernel

Each shape is checked once against an fp32 product, then both GEMMs are timed with CUDA events
over ``--iters`` launches after 3 warm-up launches; one JSON line per shape. The default shapes
are the per-rank GEMMs of the TP=8 Llama MLP (X [8192, 8192], W_up shard [8192, 3584]) and a
square one.
"""
from __future__ import annotations

import argparse
import os
import sys


def _time(fn, iters: int) -> float:
    import torch
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--shapes", default="8192x3584x8192:silu,8192x8192x3584,4096x4096x4096",
                   help="comma list of MxNxK[:silu]")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--out", default="", help="also append the records to this JSON-lines file")
    p.add_argument("--variants", default="",
                   help="also time (and check) each shape under these environment variants, e.g. "
                        "'BCCL_GEMM_BN=224,BCCL_GEMM_BN=auto,BCCL_GEMM_PAIR=0'")
    args = p.parse_args(argv)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import torch
    from originccl_b200.ops import gemm
    from originccl_b200.utils.results import ResultLog

    log = ResultLog("gemm_bench", args.out)

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    rc = 0
    for spec in args.shapes.split(","):
        dims, _, act = spec.partition(":")
        m, n, k = (int(x) for x in dims.split("x"))
        act = act or None
        a = (torch.randn(m, k, device="cuda", generator=g) * 0.5).bfloat16()
        w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16()
        y = gemm.gemm(a, w, act)
        ref = a.float() @ w.float().t()
        if act:
            ref = torch.nn.functional.silu(ref)
        err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
        del ref
        ok = err < 2e-2 and gemm.check_error() == 0
        rc |= 0 if ok else 1
        ours = _time(lambda: gemm.gemm(a, w, act, out=y), args.iters)
        cub = _time(lambda: torch.matmul(a, w.t()), args.iters)
        fl = 2.0 * m * n * k
        variants = {}
        for var in filter(None, args.variants.split(",")):
            key, _, val = var.partition("=")
            saved = os.environ.get(key)
            os.environ[key] = val
            yv = gemm.gemm(a, w, act)
            refv = a.float() @ w.float().t()
            if act:
                refv = torch.nn.functional.silu(refv)
            errv = ((yv.float() - refv).abs().max() / refv.abs().max()).item()
            del refv
            okv = errv < 2e-2 and gemm.check_error() == 0
            rc |= 0 if okv else 1
            tv = _time(lambda: gemm.gemm(a, w, act, out=yv), args.iters)
            variants[var] = {"kernel": gemm.kernel_name(m, n), "ms": round(tv, 4),
                             "tflops": round(fl / tv / 1e9, 1), "ok": okv}
            if saved is None:
                os.environ.pop(key, None)
            else:
                os.environ[key] = saved
        log({"shape": spec, "kernel": gemm.kernel_name(m, n), "ours_ms": round(ours, 4),
             "ours_tflops": round(fl / ours / 1e9, 1), "cublas_ms": round(cub, 4),
             "cublas_tflops": round(fl / cub / 1e9, 1), "rel_err": round(err, 5), "ok": ok,
             "variants": variants})
    log.close()
    return rc


if __name__ == "__main__":
    sys.exit(main())
