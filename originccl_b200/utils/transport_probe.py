"""Raw transport bandwidth over NVLink peer memory and NVSwitch multicast.

Parity: the reference's transport probes (OriginCCL tests/benchmark/test_rdma_zc_benchmark.cpp,
rdma_write_lat.cpp, rdma_pingpong.cpp) measure the byte movers below its collectives. Here the
movers are SM loads/stores to a peer's mapped memory and multimem stores, so rank 0 runs a copy
kernel with the destination (write), the source (read) or the multicast address in use while
every other rank idles at a barrier. Run one rank per GPU::

    torchrun --nproc-per-node 2 -m originccl_b200.utils.transport_probe --bytes 256M
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--bytes", default="256M")
    p.add_argument("--ctas", default="16,32,64,148,296")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--all-ranks", action="store_true",
                   help="every rank probes at the same time (rank r targets rank r+1): bidirectional traffic")
    args = p.parse_args(argv)
    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import originccl_b200 as occl
    from originccl_b200 import _native
    from originccl_b200.utils.sweep import parse_size

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    comm = occl.init_from_store(dist.distributed_c10d._get_default_store(), rank, world, device=local,
                                buffer_bytes=1 << 30)
    lib = _native.lib()
    nbytes = parse_size(args.bytes)
    peer = (rank + 1) % world if args.all_ranks else (1 if world > 1 else 0)
    modes = {0: "local_copy", 1: "peer_write", 2: "peer_read", 3: "multimem_st"}
    for mode, name in modes.items():
        if mode == 3 and not comm.nvls_enabled:
            continue
        for ctas in [int(c) for c in args.ctas.split(",")]:
            dist.barrier()
            if rank == 0 or args.all_ranks:
                gbs = lib.bcclDebugBandwidth(comm._h, mode, peer, nbytes, ctas, args.iters)
                if rank == 0:
                    print(json.dumps({"probe": name, "bytes": nbytes, "ctas": ctas, "gbs": round(gbs, 1), "peer": peer,
                                      "ranks": world, "all_ranks": args.all_ranks}), flush=True)
            dist.barrier()
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
