"""Device collective cases, run inside each rank process by the GPU tests.

Inputs are seeded per rank; the oracle recomputes every rank's input on the host and reduces in
float64, so a case needs no data from other ranks. Integer and 1/8-multiple floating inputs give
exact expected values; bf16/fp16 use tolerances.
"""
from __future__ import annotations

import os
from typing import Dict, List, Tuple

import numpy as np

DTYPES = ["float32", "float64", "int32", "int64", "bfloat16", "float16"]


def _torch_dtype(name: str):
    import torch
    return getattr(torch, name)


def rank_input(rank: int, n: int, dtype: str, seed: int = 0):
    """Exact-friendly values: multiples of 1/8 in [-8, 8) for floats, small ints for ints."""
    import torch
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    v = torch.randint(-64, 64, (n,), generator=g, dtype=torch.int64)
    if dtype.startswith("int"):
        return v.to(_torch_dtype(dtype))
    return (v.double() / 8.0).to(_torch_dtype(dtype))


def oracle(op: str, inputs: List, world: int):
    import torch
    stack = torch.stack([x.double() for x in inputs])
    if op in ("sum", "avg"):
        r = stack.sum(0)
    elif op == "max":
        r = stack.max(0).values
    else:
        r = stack.min(0).values
    if op == "avg":
        if inputs[0].dtype in (torch.int32, torch.int64):
            r = torch.div(r, world, rounding_mode="trunc")
        else:
            r = r / world
    return r


def _tol(dtype: str) -> Tuple[float, float]:
    return {"bfloat16": (1.6e-2, 1e-1), "float16": (2e-3, 2e-2)}.get(dtype, (0.0, 0.0))


def _close(got, exp, dtype: str, what: str) -> None:
    import torch
    rtol, atol = _tol(dtype)
    got = got.double().cpu()
    exp = exp.double().cpu()
    if rtol == 0 and atol == 0:
        if not torch.equal(got, exp):
            bad = (got != exp).nonzero()
            i = int(bad[0]) if bad.numel() else -1
            raise AssertionError(f"{what}: mismatch at {i}: got {got[i].item()} expected {exp[i].item()} "
                                 f"({bad.numel()} bad)")
    else:
        torch.testing.assert_close(got, exp, rtol=rtol, atol=atol, msg=lambda m: f"{what}: {m}")


OPS = {"sum": 0, "max": 1, "min": 2, "avg": 3}


def agree_state(comm, what: str) -> None:
    """Every rank's device-side sequence counters must be equal after the same calls (a rank whose
    counters drift would pass a later cross-rank barrier early or use the wrong inbox half)."""
    import torch
    if comm.world_size < 2:
        return
    mine = torch.tensor(comm.device_state(), dtype=torch.int64, device="cuda")
    allst = torch.empty(comm.world_size * mine.numel(), dtype=torch.int64, device="cuda")
    comm.all_gather(allst, mine)
    rows = allst.view(comm.world_size, -1).cpu().tolist()
    assert all(r == rows[0] for r in rows), f"device counters diverged after {what}: {rows}"
    assert rows[0][5] == 0, f"finished-CTA count left at {rows[0][5]} after {what}"


def run_suite(rank: int, world: int, sizes: List[int], algos: List[str], quick: bool = False) -> Dict:
    """Runs every collective over dtypes x ops x sizes x algorithms; returns a summary."""
    import torch

    import originccl_b200 as occl
    from originccl_b200 import Algo, ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    algo_map = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS, "ring": Algo.RING,
                "hybrid": Algo.HYBRID, "ll": Algo.LL}
    ran = 0
    used = set()
    dtypes = ["float32", "bfloat16", "int32"] if quick else DTYPES
    for n in sizes:
        for dtype in dtypes:
            td = _torch_dtype(dtype)
            inputs = [rank_input(r, n, dtype, seed=n) for r in range(world)]
            x = inputs[rank].cuda()
            # AllReduce: every op, out of place and in place, each algorithm
            for op in (["sum", "max", "avg"] if quick else ["sum", "max", "min", "avg"]):
                exp = oracle(op, inputs, world)
                for algo in algos:
                    y = torch.full((n + 1,), 7, dtype=td, device="cuda")  # sentinel after the output
                    comm.all_reduce(x, ReduceOp(OPS[op]), out=y[:n], algo=algo_map[algo])
                    used.add(comm.last_algorithm)
                    agree_state(comm, f"allreduce {dtype} {op} n={n} algo={algo}")
                    _close(y[:n], exp.to(td), dtype, f"allreduce {dtype} {op} n={n} algo={algo}")
                    assert y[n].item() == 7, "allreduce wrote past the end"
                    ran += 1
                xi = x.clone()
                comm.all_reduce(xi, ReduceOp(OPS[op]))
                _close(xi, exp.to(td), dtype, f"allreduce in-place {dtype} {op} n={n}")
                _close(x, inputs[rank].cuda(), dtype, "input changed")
            # ReduceScatter: input world*n; AllGather (each algorithm that applies: one-shot push or
            # NVLS; the others fall back to auto)
            rs_in = [rank_input(r, n * world, dtype, seed=n + 1) for r in range(world)]
            rs_x = rs_in[rank].cuda()
            for algo in algos:
                out = torch.full((n + 1,), 7, dtype=td, device="cuda")
                comm.reduce_scatter(out[:n], rs_x, algo=algo_map[algo])
                used.add("rs:" + comm.last_algorithm)
                agree_state(comm, f"reducescatter {dtype} n={n} algo={algo}")
                _close(out[:n], oracle("sum", rs_in, world)[rank * n:(rank + 1) * n].to(td), dtype,
                       f"reducescatter {dtype} n={n} algo={algo}")
                assert out[n].item() == 7, "reducescatter wrote past the end"
                ag = torch.full((n * world + 1,), 7, dtype=td, device="cuda")
                comm.all_gather(ag[:n * world], x, algo=algo_map[algo])
                used.add("ag:" + comm.last_algorithm)
                agree_state(comm, f"allgather {dtype} n={n} algo={algo}")
                _close(ag[:n * world], torch.cat(inputs).to(td), dtype, f"allgather {dtype} n={n} algo={algo}")
                assert ag[n * world].item() == 7, "allgather wrote past the end"
            _close(rs_x, rs_in[rank].cuda(), dtype, "reducescatter input changed")
            # Broadcast from the last rank, Reduce MAX to rank 0
            root = world - 1
            b = x.clone()
            comm.broadcast(b, root)
            agree_state(comm, f"broadcast {dtype} n={n}")
            _close(b, inputs[root].to(td), dtype, f"broadcast {dtype} n={n}")
            for algo in algos:
                r_out = torch.empty(n, dtype=td, device="cuda") if rank == 0 else None
                comm.reduce(x, 0, ReduceOp.MAX, out=r_out, algo=algo_map[algo])
                if rank == 0:
                    _close(r_out, oracle("max", inputs, world).to(td), dtype, f"reduce {dtype} n={n} algo={algo}")
            ran += 4
    # A group of many small collectives runs as one batched launch.
    before = comm.kernel_launches
    tensors = [rank_input(rank, 1024 + 3 * i, "float32", seed=i).cuda() for i in range(64)]
    outs = [torch.empty_like(t) for t in tensors]
    with comm.group():
        for t, o in zip(tensors, outs):
            comm.all_reduce(t, out=o, scale=0.5)
    launches = comm.kernel_launches - before
    for i, o in enumerate(outs):
        exp = oracle("sum", [rank_input(r, 1024 + 3 * i, "float32", seed=i) for r in range(world)], world) * 0.5
        _close(o, exp.float(), "float32", f"group item {i}")
    nvls = comm.nvls_enabled
    comm.destroy()
    return {"ran": ran, "algorithms": sorted(used), "group_launches": launches, "nvls": nvls}


def run_p2p(rank: int, world: int) -> Dict:
    import torch

    import originccl_b200 as occl
    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    n = (4 << 20) // 4
    s = torch.full((n,), float(rank), device="cuda")
    r = torch.empty(n, device="cuda")
    with comm.group():
        comm.send(s, (rank + 1) % world)
        comm.recv(r, (rank - 1) % world)
    assert torch.all(r == float((rank - 1) % world)).item()
    comm.destroy()
    return {"ok": True}


def run_p2p_native(rank: int, world: int) -> Dict:
    """Send/Recv on the native kernel (BCCL_P2P_NATIVE=1 in the environment): a ring exchange
    and a both-ways exchange with every peer, several operations per pair (FIFO), odd and
    unaligned sizes, sizes of many chunks, repeated so the per-channel counters carry over."""
    import torch

    import originccl_b200 as occl
    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    algos = set()
    for it in range(3):
        sizes = [1, 4097, (3 << 20) // 4 + 3, 65536 // 4]
        outs = []
        with comm.group():
            for j, n in enumerate(sizes):
                s = torch.arange(n, device="cuda", dtype=torch.float32) + 1000.0 * (rank * 10 + j) + it
                r = torch.full((n,), -1.0, device="cuda")
                comm.send(s, nxt)
                comm.recv(r, prv)
                outs.append((r, n, j))
        algos.add(comm.last_algorithm)
        for r, n, j in outs:
            want = torch.arange(n, device="cuda", dtype=torch.float32) + 1000.0 * (prv * 10 + j) + it
            assert torch.equal(r, want), (it, j)
        # every peer both ways, bf16 at an odd element offset (2-byte aligned buffers)
        base = torch.zeros(world * 70001 + 1, device="cuda", dtype=torch.bfloat16)
        got = torch.full((world * 70001 + 1,), -1.0, device="cuda", dtype=torch.bfloat16)
        for q in range(world):
            base[1 + q * 70001:1 + (q + 1) * 70001] = float(rank * 8 + q)
        with comm.group():
            for q in range(world):
                if q == rank:
                    continue
                comm.send(base[1 + q * 70001:1 + (q + 1) * 70001], q)
                comm.recv(got[1 + q * 70001:1 + (q + 1) * 70001], q)
        for q in range(world):
            if q != rank:
                assert torch.all(got[1 + q * 70001:1 + (q + 1) * 70001] == float(q * 8 + rank)).item(), (it, q)
    # all_to_all: one Send/Recv group with every peer
    n = 3 * 65536 + 5
    x = torch.cat([torch.full((n,), float(rank * 10 + q), device="cuda") for q in range(world)])
    out = torch.empty_like(x)
    comm.all_to_all(out, x)
    want = torch.cat([torch.full((n,), float(q * 10 + rank), device="cuda") for q in range(world)])
    assert torch.equal(out, want)
    comm.destroy()
    return {"algorithms": sorted(algos)}


def run_timeout_probe(rank: int, world: int) -> Dict:
    """Rank 1 never launches its collective; rank 0's bounded wait must expire and report an
    error status while the GPU context stays usable."""
    import torch

    import originccl_b200 as occl
    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=500, enable_nvls=False, enable_nccl_p2p=False)
    x = torch.ones(1024, device="cuda")
    result = {}
    if rank == 0:
        try:
            comm.all_reduce(x)
            result["raised"] = False
        except occl.BcclError as e:
            result["raised"] = True
            result["msg"] = str(e)
        # The context still works after the failed collective.
        z = torch.arange(10, device="cuda").sum().item()
        result["context_ok"] = z == 45
    comm.barrier()  # host-side: rank 1 leaves only after rank 0 has finished waiting
    comm.destroy()
    return result


def run_mixed_sequence(rank: int, world: int, steps: int = 60) -> Dict:
    """Random interleaving of every kernel kind and size (same sequence on every rank): checks
    that consecutive launches of different algorithms never corrupt each other's staging."""
    import random

    import torch

    import originccl_b200 as occl
    from originccl_b200 import Algo, ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, timeout_ms=20000)  # async: enqueue back to back
    rng = random.Random(99)
    pending = []
    algos = [Algo.AUTO, Algo.ONESHOT, Algo.TWOSHOT, Algo.NVLS, Algo.RING]
    for i in range(steps):
        n = rng.choice([3, 1000, 65536 + 7, 1 << 20, (5 << 20) + 11])
        kind = rng.choice(["ar", "ar", "ag", "rs", "bc", "red"])
        inputs = [rank_input(r, n, "float32", seed=i) for r in range(world)]
        x = inputs[rank].cuda()
        if kind == "ar":
            y = torch.empty_like(x)
            comm.all_reduce(x, out=y, algo=rng.choice(algos))
            pending.append((y, oracle("sum", inputs, world).float(), f"ar step {i}"))
        elif kind == "ag":
            y = torch.empty(n * world, device="cuda")
            comm.all_gather(y, x)
            pending.append((y, torch.cat(inputs).float(), f"ag step {i}"))
        elif kind == "rs":
            big = [rank_input(r, n * world, "float32", seed=i) for r in range(world)]
            y = torch.empty(n, device="cuda")
            comm.reduce_scatter(y, big[rank].cuda())
            pending.append((y, oracle("sum", big, world)[rank * n:(rank + 1) * n].float(), f"rs step {i}"))
        elif kind == "bc":
            root = i % world
            y = x.clone()
            comm.broadcast(y, root, algo=rng.choice([Algo.AUTO, Algo.NVLS, Algo.ONESHOT]))
            pending.append((y, inputs[root].float(), f"bc step {i}"))
        else:
            root = (i + 1) % world
            y = torch.empty_like(x) if rank == root else None
            comm.reduce(x, root, ReduceOp.SUM, out=y, algo=rng.choice([Algo.AUTO, Algo.NVLS, Algo.ONESHOT]))
            if rank == root:
                pending.append((y, oracle("sum", inputs, world).float(), f"reduce step {i}"))
    comm.synchronize()
    for got, exp, what in pending:
        _close(got, exp, "float32", what)
    comm.destroy()
    return {"checked": len(pending)}


def run_tp(rank: int, world: int, ms: int = 256, k: int = 512, nf: int = 384, hd: int = 512, calls: int = 3) -> Dict:
    """Fused AllGather->GEMM(SiLU) and GEMM->ReduceScatter against an fp32 oracle rebuilt from seeds."""
    import torch

    import originccl_b200 as occl
    from originccl_b200.ops import tp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)

    def shard(r, c):
        g = torch.Generator(device="cuda").manual_seed(1000 * c + r)
        return (torch.randn(ms, k, device="cuda", generator=g) * 0.5).bfloat16()

    def w_up(r):
        g = torch.Generator(device="cuda").manual_seed(50000 + r)
        return (torch.randn(nf, k, device="cuda", generator=g) * 0.05).bfloat16()

    def w_down(r):
        g = torch.Generator(device="cuda").manual_seed(60000 + r)
        return (torch.randn(hd, nf, device="cuda", generator=g) * 0.05).bfloat16()

    worst_ag = worst_rs = 0.0
    for c in range(calls):
        x = shard(rank, c)
        y = tp.all_gather_gemm(comm, x, w_up(rank), "silu")
        comm.synchronize()
        full = torch.cat([shard(q, c) for q in range(world)]).float()
        ref = torch.nn.functional.silu(full @ w_up(rank).float().t())
        err = ((y.float() - ref).abs().max() / ref.abs().max()).item()
        worst_ag = max(worst_ag, err)
        assert err < 2e-2, f"all_gather_gemm call {c}: rel err {err}"
        # GEMM->ReduceScatter with h = this call's y (same on... each rank has its own h)
        out = tp.gemm_reduce_scatter(comm, y, w_down(rank))
        comm.synchronize()
        acc = torch.zeros(ms * world, hd, device="cuda")
        for q in range(world):
            fq = torch.cat([shard(p, c) for p in range(world)]).float()
            hq = torch.nn.functional.silu(fq @ w_up(q).float().t()).bfloat16().float()
            acc += hq @ w_down(q).float().t()
        ref2 = acc[rank * ms:(rank + 1) * ms]
        err2 = ((out.float() - ref2).abs().max() / ref2.abs().max()).item()
        worst_rs = max(worst_rs, err2)
        assert err2 < 3e-2, f"gemm_reduce_scatter call {c}: rel err {err2}"
    comm.destroy()
    return {"ag_err": worst_ag, "rs_err": worst_rs}


def run_dp(rank: int, world: int, hidden: int = 256, steps: int = 2) -> Dict:
    """Data-parallel sync on the GPU (buckets on a side stream during backward, small tensors
    as one group) against gradients averaged locally from every rank's batch."""
    import torch

    import originccl_b200 as occl
    from originccl_b200.models import TinyLlamaStack
    from originccl_b200.parallel.data_parallel import DataParallelSync, GradBuckets

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, timeout_ms=20000)

    def grads_of(r: int):
        m = TinyLlamaStack(hidden=hidden, ffn=3 * hidden, layers=2, seed=5).cuda()
        g = torch.Generator(device="cuda").manual_seed(300 + r)
        m(torch.randn(32, hidden, device="cuda", generator=g)).pow(2).mean().backward()
        return {n: p.grad.detach().clone() for n, p in m.named_parameters()}

    model = TinyLlamaStack(hidden=hidden, ffn=3 * hidden, layers=2, seed=5).cuda()
    grads = GradBuckets(model.named_parameters(), bucket_bytes=64 << 10, small_bytes=4096)
    dp = DataParallelSync(comm, grads)
    dp.attach()
    g = torch.Generator(device="cuda").manual_seed(300 + rank)
    x = torch.randn(32, hidden, device="cuda", generator=g)
    for _ in range(steps):
        grads.zero_()
        model(x).pow(2).mean().backward()
        dp.finish()
    torch.cuda.synchronize()
    expect = [grads_of(r) for r in range(world)]
    worst = 0.0
    for n, p in model.named_parameters():
        ref = sum(e[n] for e in expect) / world
        err = ((p.grad - ref).abs().max() / ref.abs().max().clamp_min(1e-12)).item()
        worst = max(worst, err)
        assert err < 1e-4, f"{n}: relative error {err}"
    registered = dp.registered
    dp.close()
    comm.destroy()
    return {"buckets": grads.num_buckets, "small": len(grads.small_idx), "worst": worst, "registered": registered}


def run_zero_copy(rank: int, world: int) -> Dict:
    """Collectives on symmetric (multicast-bound) buffers through the zero-copy NVLS kernel:
    AllReduce in place and out of place, AllGather into a symmetric output, ReduceScatter from a
    symmetric input, against a float64 oracle."""
    import torch

    import originccl_b200 as occl
    from originccl_b200 import Algo, ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    if not comm.nvls_enabled:
        comm.destroy()
        return {"skipped": True}
    used = set()
    for dtype, n in (("float32", 4096), ("float32", (1 << 20) + 4), ("bfloat16", 3 << 18)):
        td = getattr(torch, dtype)
        inputs = [rank_input(r, n, dtype, seed=n) for r in range(world)]
        src = comm.symmetric_empty((n,), td)
        dst = comm.symmetric_empty((n,), td)
        src.copy_(inputs[rank].cuda())
        torch.cuda.synchronize()  # the communicator's own stream does not wait for torch's
        comm.all_reduce(src, ReduceOp.SUM, out=dst, algo=Algo.NVLS)
        used.add(comm.last_algorithm)
        _close(dst, oracle("sum", inputs, world).to(td), dtype, f"zero-copy {dtype} n={n}")
        comm.all_reduce(src, ReduceOp.AVG, algo=Algo.NVLS)  # in place
        _close(src, oracle("avg", inputs, world).to(td), dtype, f"zero-copy in place {dtype} n={n}")
    # AllGather into a symmetric output, ReduceScatter from a symmetric input.
    for dtype, n in (("float32", 1024), ("bfloat16", 5 << 16)):
        td = getattr(torch, dtype)
        blocks = [rank_input(r, n, dtype, seed=n + 1) for r in range(world)]
        gathered = comm.symmetric_empty((world * n,), td)
        mine = blocks[rank].cuda()
        torch.cuda.synchronize()
        comm.all_gather(gathered, mine)
        used.add(comm.last_algorithm)
        _close(gathered, torch.cat(blocks).to(td), dtype, f"zero-copy all_gather {dtype} n={n}")
        full = [rank_input(r, world * n, dtype, seed=n + 2) for r in range(world)]
        src = comm.symmetric_empty((world * n,), td)
        src.copy_(full[rank].cuda())
        torch.cuda.synchronize()
        shard = torch.empty(n, dtype=td, device="cuda")
        comm.reduce_scatter(shard, src, ReduceOp.SUM)
        used.add(comm.last_algorithm)
        want = oracle("sum", full, world)[rank * n:(rank + 1) * n].to(td)
        _close(shard, want, dtype, f"zero-copy reduce_scatter {dtype} n={n}")
    comm.destroy()
    return {"algorithms": sorted(used)}


def run_graph(rank: int, world: int) -> Dict:
    """Collectives captured into CUDA graphs and replayed: a small AllReduce (push engine), a
    group of three collectives (one batched kernel) and a large AllReduce (pipelined kernels),
    each replayed several times with new input values written between replays; every replay is
    checked against the float64 oracle. Replays run without the host, so this also checks that
    the device-side sequence numbers carry the cross-rank synchronisation."""
    import torch

    import originccl_b200 as occl
    from originccl_b200 import ReduceOp
    from originccl_b200.utils.graphs import capture

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, timeout_ms=20000)  # stream-ordered
    small, large = 3000, (24 << 20) // 4 + 12
    x = torch.empty(small, device="cuda")
    y = torch.empty(small, device="cuda")
    a = torch.empty(1000, device="cuda")
    g_in = torch.empty(777, device="cuda")
    g_out = torch.empty(777 * world, device="cuda")
    rs_in = torch.empty(512 * world, device="cuda")
    rs_out = torch.empty(512, device="cuda")
    big = torch.empty(large, device="cuda")
    big_out = torch.empty(large, device="cuda")

    def fill(seed: int):
        ins = {}
        for k, (name, t, n) in enumerate((("x", x, small), ("a", a, 1000), ("g", g_in, 777),
                                          ("rs", rs_in, 512 * world), ("big", big, large))):
            per_rank = [rank_input(r, n, "float32", seed=seed * 10 + k) for r in range(world)]
            t.copy_(per_rank[rank].cuda())
            ins[name] = per_rank
        return ins

    def step():
        comm.all_reduce(x, ReduceOp.SUM, out=y)
        with comm.group():
            comm.all_reduce(a, ReduceOp.MAX)
            comm.all_gather(g_out, g_in)
            comm.reduce_scatter(rs_out, rs_in, ReduceOp.SUM)
        comm.all_reduce(big, ReduceOp.SUM, out=big_out, scale=0.5)

    fill(0)
    graph = capture(step, repeat=1, warmup=2)
    launches = comm.kernel_launches
    for it in range(1, 5):
        ins = fill(it)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        comm.synchronize()  # reports device-side failures of the replay
        _close(y, oracle("sum", ins["x"], world), "float32", f"graph replay {it}: small all_reduce")
        _close(a, oracle("max", ins["a"], world), "float32", f"graph replay {it}: grouped all_reduce max")
        _close(g_out, torch.cat(ins["g"]), "float32", f"graph replay {it}: grouped all_gather")
        _close(rs_out, oracle("sum", ins["rs"], world)[rank * 512:(rank + 1) * 512], "float32",
               f"graph replay {it}: grouped reduce_scatter")
        _close(big_out, oracle("sum", ins["big"], world) * 0.5, "float32", f"graph replay {it}: large all_reduce")
    host_launches = comm.kernel_launches - launches  # replays do not go through the library
    del graph
    comm.destroy()
    return {"replays": 4, "host_launches_during_replays": host_launches}


def run_registered(rank: int, world: int) -> Dict:
    """Ordinary PyTorch CUDA tensors registered with the communicator (CUDA IPC): AllReduce
    (out of place, in place, AVG, bf16 with a scale), AllGather, ReduceScatter and views of one
    registered flat buffer at the same offsets on every rank (gradient buckets) run over peer
    memory without staging; checked against the float64 oracle, with a sentinel after each
    output. Below the size threshold the staged kernels run on the same buffers."""
    import torch

    import originccl_b200 as occl
    from originccl_b200 import ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    used = set()
    n = (3 << 20) // 4 + 8                   # 3 MiB of fp32, above the 1 MiB threshold
    ins = [rank_input(r, n, "float32", seed=5) for r in range(world)]
    x = ins[rank].cuda()
    y = torch.full((n + 4,), 77.0, device="cuda")  # 16-byte sentinel tail
    comm.register(x)
    comm.register(y)
    comm.all_reduce(x, ReduceOp.SUM, out=y[:n])
    used.add(comm.last_algorithm)
    _close(y[:n], oracle("sum", ins, world), "float32", "registered all_reduce")
    assert bool((y[n:] == 77.0).all()), "registered all_reduce wrote past the output"
    comm.all_reduce(x, ReduceOp.AVG)           # in place
    _close(x, oracle("avg", ins, world), "float32", "registered all_reduce in place avg")
    # AllGather into / ReduceScatter from registered buffers.
    m = (1 << 20) // 4
    blocks = [rank_input(r, m, "float32", seed=6) for r in range(world)]
    gathered = torch.empty(world * m, device="cuda")
    comm.register(gathered)
    comm.all_gather(gathered, blocks[rank].cuda())
    used.add(comm.last_algorithm)
    _close(gathered, torch.cat(blocks), "float32", "registered all_gather")
    full = [rank_input(r, world * m, "float32", seed=7) for r in range(world)]
    rs_in = full[rank].cuda()
    comm.register(rs_in)
    shard = torch.empty(m, device="cuda")
    comm.reduce_scatter(shard, rs_in, ReduceOp.MAX)
    used.add(comm.last_algorithm)
    _close(shard, oracle("max", full, world)[rank * m:(rank + 1) * m], "float32", "registered reduce_scatter max")
    # bf16 buckets: views of one registered flat buffer, scaled mean as in gradient sync.
    nb, per = 4, (1 << 20)
    grads = [rank_input(r, nb * per, "bfloat16", seed=8) for r in range(world)]
    flat = grads[rank].cuda()
    comm.register(flat)
    for b in range(nb):
        comm.all_reduce(flat[b * per:(b + 1) * per], ReduceOp.SUM, scale=1.0 / world)
        used.add(comm.last_algorithm)
    _close(flat, (oracle("sum", grads, world) / world).to(torch.bfloat16), "bfloat16", "registered bf16 buckets")
    # A small message on registered memory still takes the batched push kernel.
    comm.all_reduce(flat[:256], ReduceOp.MAX)
    small_algo = comm.last_algorithm
    for t in (flat, rs_in, gathered, y, x):
        comm.deregister(t)
    comm.destroy()
    return {"algorithms": sorted(used), "small_algorithm": small_algo}


def run_fuzz(rank: int, world: int, seed: int, n_ops: int) -> Dict:
    """Device counterpart of the host path's random sequences: every rank draws the same
    sequence of collectives (kind, dtype, op, size up to 48 MiB, root, algorithm, in place or
    not, alone or in groups with Send/Recv) and checks each result against the float64 oracle
    with a sentinel after every output. Buffers stay alive until their group has run."""
    import numpy as np
    import torch

    import originccl_b200 as occl
    from originccl_b200 import Algo, ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=30000)
    rng = np.random.default_rng(seed)
    algos = {"auto": Algo.AUTO, "oneshot": Algo.ONESHOT, "twoshot": Algo.TWOSHOT, "nvls": Algo.NVLS, "ring": Algo.RING}
    checks, keep, used = [], [], set()
    done = 0

    def one(i: int, grouped: bool):
        kind = str(rng.choice(["allreduce", "reduce", "broadcast", "allgather", "reducescatter", "sendrecv"]))
        dtype = str(rng.choice(["float32", "bfloat16", "float16", "int32", "int64", "float64"]))
        op = str(rng.choice(list(OPS)))
        if dtype == "float16" and op == "avg":
            op = "sum"
        n = int(rng.choice([0, 1, 5, 1000, 4099, 65536 + 8, 300001, 1 << 20, (6 << 20) + 4, 12 << 20]))
        root = int(rng.integers(0, world))
        algo = str(rng.choice(list(algos))) if not grouped else "auto"
        inplace = bool(rng.integers(0, 2))
        td = _torch_dtype(dtype)
        tag = f"op {i} {kind} {dtype} {op} n={n} root={root} algo={algo} inplace={inplace}"
        ins = [rank_input(r, n, dtype, seed=seed * 1000 + i) for r in range(world)]
        x = ins[rank].cuda()
        out = torch.full((n + 1,), 7, dtype=td, device="cuda")
        keep.extend([x, out])
        sentinel = lambda: (out[n].item() == 7) or (_ for _ in ()).throw(AssertionError(tag + ": wrote past the end"))  # noqa: E731
        if kind == "broadcast" and rank == root:
            out[:n].copy_(x)
        # The communicator runs on its own stream: inputs written on torch's stream must be done.
        torch.cuda.synchronize()
        if kind == "allreduce":
            if inplace:
                comm.all_reduce(x, ReduceOp(OPS[op]), algo=algos[algo])
                checks.append(lambda: _close(x, oracle(op, ins, world).to(td), dtype, tag))
            else:
                comm.all_reduce(x, ReduceOp(OPS[op]), out=out[:n], algo=algos[algo])
                checks.append(lambda: (_close(out[:n], oracle(op, ins, world).to(td), dtype, tag), sentinel()))
        elif kind == "reduce":
            comm.reduce(x, root, ReduceOp(OPS[op]), out=out[:n] if rank == root else None, algo=algos[algo])
            if rank == root:
                checks.append(lambda: (_close(out[:n], oracle(op, ins, world).to(td), dtype, tag), sentinel()))
        elif kind == "broadcast":
            comm.broadcast(out[:n], root, algo=algos[algo])
            checks.append(lambda: (_close(out[:n], ins[root].to(td), dtype, tag), sentinel()))
        elif kind == "allgather":
            g = torch.full((n * world + 1,), 7, dtype=td, device="cuda")
            keep.append(g)
            torch.cuda.synchronize()
            comm.all_gather(g[:n * world], x)
            checks.append(lambda: (_close(g[:n * world], torch.cat(ins).to(td), dtype, tag),
                                   (g[n * world].item() == 7) or (_ for _ in ()).throw(AssertionError(tag))))
        elif kind == "reducescatter":
            full = [rank_input(r, n * world, dtype, seed=seed * 1000 + i + 7) for r in range(world)]
            xi = full[rank].cuda()
            keep.append(xi)
            torch.cuda.synchronize()
            comm.reduce_scatter(out[:n], xi, ReduceOp(OPS[op]))
            checks.append(lambda: (_close(out[:n], oracle(op, full, world)[rank * n:(rank + 1) * n].to(td), dtype, tag),
                                   sentinel()))
        elif world > 1:
            nxt, prv = (rank + 1) % world, (rank - 1) % world
            if grouped:
                comm.send(x, nxt)
                comm.recv(out[:n], prv)
            else:
                with comm.group():
                    comm.send(x, nxt)
                    comm.recv(out[:n], prv)
            checks.append(lambda: (_close(out[:n], ins[prv].to(td), dtype, tag), sentinel()))

    i = 0
    while i < n_ops:
        mode = int(rng.integers(0, 3))
        if mode == 0:
            one(i, False)
            i += 1
            used.add(comm.last_algorithm)
        else:
            k = int(rng.integers(2, 7))
            comm.group_start()
            if mode == 2:
                comm.group_start()
            for _ in range(k):
                one(i, True)
                i += 1
            if mode == 2:
                comm.group_end()
            comm.group_end()
        torch.cuda.synchronize()
        for c in checks:
            c()
        done += len(checks)
        checks.clear()
        keep.clear()
    comm.destroy()
    return {"checked": done, "algorithms": sorted(used)}


def run_split_device(rank: int, world: int) -> Dict:
    """Device communicators split like MPI_Comm_split: all ranks in one color (reversed), then
    every rank alone; AllReduce runs in each child against the oracle."""
    import torch

    import originccl_b200 as occl
    from originccl_b200 import ReduceOp

    dev = rank % torch.cuda.device_count()
    torch.cuda.set_device(dev)
    comm = occl.init_from_env(device=dev, blocking=True, timeout_ms=20000)
    both = comm.split(0, key=-rank)
    alone = comm.split(rank)
    ins = [rank_input(r, 5000, "float32", seed=9) for r in range(world)]
    x = ins[rank].cuda()
    y = torch.empty_like(x)
    both.all_reduce(x, ReduceOp.SUM, out=y)
    _close(y, oracle("sum", ins, world), "float32", "split: all ranks")
    alone.all_reduce(x, ReduceOp.SUM, out=y)
    _close(y, ins[rank], "float32", "split: one rank")
    res = {"both_rank": both.rank, "alone_size": alone.world_size}
    alone.destroy()
    both.destroy()
    comm.destroy()
    return res
