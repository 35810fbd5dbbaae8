"""Runs one kernel of the library on a small single-GPU case (for ncu captures and spot checks).

    python -m originccl_b200.utils.kernel_case gemm --m 4096 --n 3584 --k 4096 --reps 3
    python -m originccl_b200.utils.kernel_case allreduce --bytes 256M --reps 3

Each case checks its result once against PyTorch, then runs the kernel ``--reps`` more times,
and exits non-zero on a mismatch.
"""
from __future__ import annotations

import argparse
import os
import sys


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("case", choices=["gemm", "allreduce", "noalloc"])
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=3584)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--act", default="none", choices=["none", "silu"])
    p.add_argument("--bytes", default="256M")
    p.add_argument("--reps", type=int, default=3)
    args = p.parse_args(argv)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import torch

    torch.cuda.set_device(0)
    if args.case == "gemm":
        from originccl_b200.ops import gemm
        g = torch.Generator(device="cuda").manual_seed(0)
        a = (torch.randn(args.m, args.k, device="cuda", generator=g) * 0.5).bfloat16()
        w = (torch.randn(args.n, args.k, device="cuda", generator=g) * 0.05).bfloat16()
        act = None if args.act == "none" else args.act
        y = gemm.gemm(a, w, act)
        ref = a.float() @ w.float().t()
        if act:
            ref = torch.nn.functional.silu(ref)
        err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
        if err > 2e-2 or gemm.check_error() != 0:
            print(f"gemm mismatch: rel err {err}")
            return 1
        for _ in range(args.reps):
            gemm.gemm(a, w, act, out=y)
        torch.cuda.synchronize()
        print(f"gemm ok rel_err={err:.4g}")
        return 0
    from originccl_b200.utils.sweep import parse_size
    import originccl_b200 as occl
    n = parse_size(args.bytes) // 4
    comm = occl.Communicator().init(0, 1, None, device=0, blocking=True)
    x = torch.rand(n, device="cuda")
    y = torch.empty_like(x)
    comm.all_reduce(x, out=y, scale=0.5)
    if not torch.equal(y, x * 0.5):
        print("allreduce mismatch")
        return 1
    for _ in range(args.reps):
        comm.all_reduce(x, out=y, scale=0.5)
    comm.destroy()
    print("allreduce ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
