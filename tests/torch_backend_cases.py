"""torch.distributed "bccl" backend cases (CPU tensors -> the host communicator)."""
from __future__ import annotations

import datetime
import os
from typing import Dict


def _init(rank: int, world: int):
    import torch.distributed as dist
    import originccl_b200.torch_backend  # noqa: F401  (registers "bccl")
    path = os.environ["BCCL_ID_FILE"] + ".torchstore"
    dist.init_process_group("bccl", init_method=f"file://{path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def run_collectives(rank: int, world: int) -> Dict:
    import torch
    dist = _init(rank, world)
    for op, ref in ((dist.ReduceOp.SUM, sum(range(1, world + 1))), (dist.ReduceOp.MAX, world),
                    (dist.ReduceOp.MIN, 1), (dist.ReduceOp.AVG, sum(range(1, world + 1)) / world)):
        x = torch.full((33,), float(rank + 1))
        dist.all_reduce(x, op=op)
        assert torch.all(x == ref), (op, x[:3])
    y = torch.arange(7.0) if rank == world - 1 else torch.zeros(7)
    dist.broadcast(y, world - 1)
    assert torch.equal(y, torch.arange(7.0))
    z = torch.full((5,), float(rank))
    dist.reduce(z, 0)
    if rank == 0:
        assert torch.all(z == sum(range(world)))
    outs = [torch.empty(3) for _ in range(world)]
    dist.all_gather(outs, torch.full((3,), float(rank)))
    assert all(torch.all(o == r) for r, o in enumerate(outs))
    flat = torch.empty(world * 4)
    dist.all_gather_into_tensor(flat, torch.full((4,), float(rank)))
    assert torch.equal(flat, torch.arange(world, dtype=torch.float32).repeat_interleave(4))
    rs = torch.empty(2)
    dist.reduce_scatter(rs, [torch.full((2,), float(r + rank)) for r in range(world)])
    assert torch.all(rs == sum(q + rank for q in range(world)))
    rt = torch.empty(3)
    dist.reduce_scatter_tensor(rt, torch.arange(3.0 * world))
    assert torch.equal(rt, world * torch.arange(3.0 * rank, 3.0 * (rank + 1)))
    if world > 1:
        nxt, prv = (rank + 1) % world, (rank - 1) % world
        s = torch.full((9,), float(rank))
        r = torch.empty(9)
        ops = [dist.P2POp(dist.isend, s, nxt), dist.P2POp(dist.irecv, r, prv)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        assert torch.all(r == prv)
    dist.barrier()
    a2a = torch.empty(world * 5)
    dist.all_to_all_single(a2a, torch.arange(world * 5, dtype=torch.float32) + 100 * rank)
    assert torch.equal(a2a, torch.cat([torch.arange(rank * 5, rank * 5 + 5, dtype=torch.float32) + 100 * q
                                       for q in range(world)]))
    outs = [torch.empty(2, dtype=torch.int64) for _ in range(world)]
    dist.all_to_all(outs, [torch.full((2,), 10 * rank + q, dtype=torch.int64) for q in range(world)])
    assert all(torch.all(o == 10 * q + rank) for q, o in enumerate(outs))
    # Uneven splits (rows of dim 0): rank r sends (r + q) % 3 + 1 rows of 4 to rank q; its
    # input block for q holds 1000 * r + 10 * q + row.
    rows = lambda a, b: (a + b) % 3 + 1  # noqa: E731  rows rank a sends to rank b
    send_rows = [rows(rank, q) for q in range(world)]
    recv_rows = [rows(q, rank) for q in range(world)]
    inp = torch.cat([torch.arange(send_rows[q], dtype=torch.float32)[:, None].repeat(1, 4) + 1000 * rank + 10 * q
                     for q in range(world)])
    out = torch.full((sum(recv_rows), 4), -1.0)
    dist.all_to_all_single(out, inp, recv_rows, send_rows)
    want = torch.cat([torch.arange(recv_rows[q], dtype=torch.float32)[:, None].repeat(1, 4) + 1000 * q + 10 * rank
                      for q in range(world)])
    assert torch.equal(out, want), (out, want)
    # Splits that do not add up to the shapes are rejected before anything is sent.
    try:
        dist.all_to_all_single(torch.empty(world), torch.empty(world), [2] * world, [1] * world)
        rejected = False
    except (ValueError, RuntimeError):
        rejected = True
    # gather / scatter to and from the last rank, with int64 values.
    root = world - 1
    gathered = [torch.empty(6, dtype=torch.int64) for _ in range(world)] if rank == root else None
    dist.gather(torch.arange(6, dtype=torch.int64) * (rank + 1), gathered, dst=root)
    if rank == root:
        assert all(torch.equal(g, torch.arange(6, dtype=torch.int64) * (q + 1)) for q, g in enumerate(gathered))
    piece = torch.empty(3)
    dist.scatter(piece, [torch.full((3,), 7.0 * q) for q in range(world)] if rank == root else None, src=root)
    assert torch.all(piece == 7.0 * rank)
    dist.destroy_process_group()
    return {"bad_splits_rejected": rejected}


def run_ddp(rank: int, world: int, hook: bool = False) -> Dict:
    import torch
    from torch.nn.parallel import DistributedDataParallel as DDP
    dist = _init(rank, world)

    def make():
        torch.manual_seed(0)
        return torch.nn.Sequential(torch.nn.Linear(16, 64), torch.nn.ReLU(), torch.nn.Linear(64, 4))

    model = make()
    ddp = DDP(model, bucket_cap_mb=0.01)  # several buckets
    if hook:
        from originccl_b200.torch_backend import AllReduceHook
        ddp.register_comm_hook(dist.group.WORLD, AllReduceHook())
    x = torch.randn(8, 16, generator=torch.Generator().manual_seed(10 + rank))
    ddp(x).pow(2).mean().backward()
    ref = None
    for r in range(world):
        m = make()
        m(torch.randn(8, 16, generator=torch.Generator().manual_seed(10 + r))).pow(2).mean().backward()
        g = [p.grad for p in m.parameters()]
        ref = g if ref is None else [a + b for a, b in zip(ref, g)]
    worst = max((p.grad - r / world).abs().max().item() for p, r in zip(model.parameters(), ref))
    assert worst < 1e-6, worst
    dist.destroy_process_group()
    return {"worst": worst}


def run_ddp_cuda(rank: int, world: int, hook: bool = False) -> Dict:
    """DDP on CUDA through the "bccl" backend (device communicator, current stream); with
    ``hook`` through AllReduceHook (fused mean; buckets of >= 64 KiB registered, zero-copy)."""
    import torch
    from torch.nn.parallel import DistributedDataParallel as DDP
    torch.cuda.set_device(rank % torch.cuda.device_count())
    dist = _init(rank, world)

    def make():
        torch.manual_seed(0)
        return torch.nn.Sequential(torch.nn.Linear(64, 256), torch.nn.ReLU(), torch.nn.Linear(256, 8)).cuda()

    model = make()
    ddp = DDP(model, bucket_cap_mb=0.05)
    h = None
    if hook:
        from originccl_b200.torch_backend import AllReduceHook
        h = AllReduceHook(min_bytes=64 << 10)
        ddp.register_comm_hook(dist.group.WORLD, h)
    g = torch.Generator(device="cuda").manual_seed(10 + rank)
    for _ in range(2 if hook else 1):  # the second step reuses the registered buckets
        model.zero_grad(set_to_none=False)
        ddp(torch.randn(32, 64, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 + rank))
            ).pow(2).mean().backward()
    torch.cuda.synchronize()
    ref = None
    for r in range(world):
        m = make()
        gr = torch.Generator(device="cuda").manual_seed(10 + r)
        m(torch.randn(32, 64, device="cuda", generator=gr)).pow(2).mean().backward()
        gl = [p.grad for p in m.parameters()]
        ref = gl if ref is None else [a + b for a, b in zip(ref, gl)]
    worst = max(((p.grad - r / world).abs().max() / (r / world).abs().max().clamp_min(1e-12)).item()
                for p, r in zip(model.parameters(), ref))
    assert worst < 1e-4, worst
    if h is not None:
        h.close()
    dist.destroy_process_group()
    return {"worst": worst}


def run_subgroups(rank: int, world: int) -> Dict:
    """dist.new_group on the "bccl" backend: each subgroup gets its own communicators (the
    group's prefixed store carries their unique ids) and collectives stay inside it."""
    import torch
    dist = _init(rank, world)
    lo, hi = list(range(world // 2)), list(range(world // 2, world))
    g_lo = dist.new_group(lo, backend="bccl")
    g_hi = dist.new_group(hi, backend="bccl")
    mine = g_lo if rank in lo else g_hi
    members = lo if rank in lo else hi
    x = torch.full((11,), float(rank + 1))
    dist.all_reduce(x, group=mine)
    assert torch.all(x == sum(r + 1 for r in members)), x[:3]
    y = torch.full((3,), float(rank))
    dist.all_reduce(y)  # the default group still spans everyone
    assert torch.all(y == sum(range(world)))
    dist.destroy_process_group()
    return {"members": members}
