"""Host-memory (CPU) collective cases, run inside each rank process.

Modeled on the reference's black-box suite (OriginCCL tests/test_common.cpp:28-399): values are
multiples of 1/8 so float and integer results compare exactly regardless of reduction order,
every output carries a sentinel element after its end, out-of-place inputs must come back
unchanged, and contract cases (count 0, missing buffer, bad root) are checked on every rank.
"""
from __future__ import annotations

from typing import Dict, List

import numpy as np

NP_DTYPES = {"float32": np.float32, "float64": np.float64, "int32": np.int32, "int64": np.int64,
             "float16": np.float16}
SENTINEL = 77


def value(rank: int, n: int, dtype: str, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed * 131 + rank)
    v = rng.integers(-64, 64, size=n)
    if dtype.startswith("int"):
        return v.astype(NP_DTYPES[dtype])
    return (v / 8.0).astype(NP_DTYPES[dtype])


def reduce_ref(op: str, arrays: List[np.ndarray], world: int) -> np.ndarray:
    st = np.stack([a.astype(np.float64) for a in arrays])
    if op == "sum":
        r = st.sum(0)
    elif op == "max":
        r = st.max(0)
    elif op == "min":
        r = st.min(0)
    else:
        r = st.sum(0)
        if np.issubdtype(arrays[0].dtype, np.integer):
            r = np.trunc(r / world)
        else:
            r = r / world
    return r.astype(arrays[0].dtype)


OPS = {"sum": 0, "max": 1, "min": 2, "avg": 3}


def _out(n: int, dtype: str) -> np.ndarray:
    return np.full(n + 1, SENTINEL, dtype=NP_DTYPES[dtype])


def _check(got: np.ndarray, exp: np.ndarray, n: int, what: str) -> None:
    assert got[n] == SENTINEL, f"{what}: wrote past the end"
    assert np.array_equal(got[:n], exp), f"{what}: mismatch (first bad {np.nonzero(got[:n] != exp)[0][:5]})"


def run_matrix(rank: int, world: int, counts: List[int], dtypes: List[str], n_channels: int = 2,
               logical_machine_size: int = 0) -> Dict:
    from originccl_b200 import ReduceOp, init_from_env
    comm = init_from_env(n_channels=n_channels, logical_machine_size=logical_machine_size, timeout_ms=30000)
    done = 0
    for n in counts:
        for dtype in dtypes:
            ins = [value(r, n, dtype, n) for r in range(world)]
            x = ins[rank].copy()
            for op in OPS:
                if dtype == "float16" and op == "avg":
                    continue
                y = _out(n, dtype)
                comm.all_reduce(x, ReduceOp(OPS[op]), out=y[:n])
                _check(y, reduce_ref(op, ins, world), n, f"allreduce {dtype} {op} n={n}")
                assert np.array_equal(x, ins[rank]), "allreduce changed its input"
                done += 1
            # in place
            xi = ins[rank].copy()
            comm.all_reduce(xi)
            assert np.array_equal(xi, reduce_ref("sum", ins, world)), f"in-place allreduce {dtype} n={n}"
            # reduce to every root with MAX
            for root in range(world):
                y = _out(n, dtype) if rank == root else None
                comm.reduce(x, root, ReduceOp.MAX, out=None if y is None else y[:n])
                if rank == root:
                    _check(y, reduce_ref("max", ins, world), n, f"reduce {dtype} root={root} n={n}")
            # broadcast from every root
            for root in range(world):
                b = ins[rank].copy()
                comm.broadcast(b, root)
                assert np.array_equal(b, ins[root]), f"broadcast {dtype} root={root} n={n}"
            # allgather (rank order) and reducescatter (N*count input)
            g = _out(n * world, dtype)
            comm.all_gather(g[:n * world], x)
            _check(g, np.concatenate(ins), n * world, f"allgather {dtype} n={n}")
            rs_in = [value(r, n * world, dtype, n + 7) for r in range(world)]
            rs = _out(n, dtype)
            comm.reduce_scatter(rs[:n], rs_in[rank].copy())
            _check(rs, reduce_ref("sum", rs_in, world)[rank * n:(rank + 1) * n], n, f"reducescatter {dtype} n={n}")
            done += 4
    info = {"ran": done, "machine_count": comm.machine_count, "local_ranks": comm.local_ranks,
            "leaders": comm.machine_leaders, "local_rank": comm.local_rank, "local_size": comm.local_size,
            "single": comm.is_single_machine, "machine_index": comm.machine_index}
    comm.destroy()
    return info


def run_contract(rank: int, world: int) -> Dict:
    """count 0 with null buffers succeeds; missing buffers, bad roots, bad peers, self peers and
    bad dtypes/ops fail on every rank before anything is queued, also inside a group."""
    import ctypes

    from originccl_b200 import BcclError, ReduceOp, init_from_env
    from originccl_b200 import _native
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    lib = _native.lib()
    h = comm._h
    null = None
    rej = 0
    # zero count, null buffers: success
    assert lib.bcclAllReduce(h, null, null, 0, 0, 0, 1.0, 0, 0, 0) == 0
    assert lib.bcclAllGather(h, null, null, 0, 0, 0, 0) == 0
    assert lib.bcclSend(h, null, 0, 0, (rank + 1) % world, 0, 0) == 0
    buf = np.zeros(8, np.float32)
    p = buf.ctypes.data
    bad = [
        lambda: lib.bcclAllReduce(h, null, p, 8, 0, 0, 1.0, 0, 0, 0),      # missing send buffer
        lambda: lib.bcclAllReduce(h, p, null, 8, 0, 0, 1.0, 0, 0, 0),      # missing recv buffer
        lambda: lib.bcclAllReduce(h, p, p, 8, 9, 0, 1.0, 0, 0, 0),         # bad dtype
        lambda: lib.bcclAllReduce(h, p, p, 8, 0, 9, 1.0, 0, 0, 0),         # bad op
        lambda: lib.bcclBroadcast(h, p, p, 8, 0, world, 0, 0, 0),          # bad root
        lambda: lib.bcclReduce(h, p, p, 8, 0, 0, -1, 0, 0, 0),             # bad root
        lambda: lib.bcclSend(h, p, 8, 0, rank, 0, 0),                      # self peer
        lambda: lib.bcclRecv(h, p, 8, 0, world, 0, 0),                     # out-of-range peer
        lambda: lib.bcclAllGather(h, p, p, (1 << 62), 0, 0, 0),            # size overflow
    ]
    for f in bad:
        assert f() != 0
        rej += 1
    # rejections inside a group are not queued: the group then runs only the valid op
    comm.group_start()
    assert bad[0]() != 0
    y = np.zeros(8, np.float32)
    x = np.full(8, rank + 1, np.float32)
    comm.all_reduce(x, out=y)
    comm.group_end()
    assert np.all(y == world * (world + 1) / 2)
    # Reduce: a non-root may pass a null recv buffer
    assert lib.bcclReduce(h, p, null if rank != 0 else p, 8, 0, 0, 0, 0, 0, 0) == 0
    # Buffer registration is a device feature; host communicators accept and ignore it.
    with comm.registered(x, y):
        comm.all_reduce(x, out=y)
    assert np.all(y == world * (world + 1) / 2)
    comm.destroy()
    return {"rejected": rej}


def run_groups(rank: int, world: int) -> Dict:
    """Nested groups: the inner GroupEnd runs nothing; the outermost runs the whole batch."""
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    xs = [np.full(1000 + i, rank + i, np.float64) for i in range(6)]
    ys = [np.zeros_like(x) for x in xs]
    comm.group_start()
    comm.all_reduce(xs[0], out=ys[0])
    comm.group_start()
    comm.all_reduce(xs[1], out=ys[1])
    comm.group_end()                     # inner: nothing runs yet
    inner_untouched = bool(np.all(ys[1] == 0))
    for i in range(2, 6):
        comm.all_reduce(xs[i], out=ys[i])
    comm.group_end()                     # outermost: everything runs
    for i in range(6):
        assert np.all(ys[i] == sum(r + i for r in range(world))), f"group item {i}"
    comm.destroy()
    return {"inner_untouched": inner_untouched}


def run_p2p(rank: int, world: int, logical_machine_size: int = 0, executor: str = "", cma: str = "") -> Dict:
    """Ring exchange in a group, FIFO for a repeated peer, a mixed 10-op group, typed messages
    around the ring-buffer capacity, a 1 MiB-per-peer mesh with receives out of order, and the
    transport each pair uses."""
    import os
    if executor:
        os.environ["BCCL_HOST_EXECUTOR"] = executor
    if cma:
        os.environ["BCCL_HOST_CMA"] = cma
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=2, logical_machine_size=logical_machine_size, timeout_ms=30000)
    nxt, prv = (rank + 1) % world, (rank - 1) % world
    for n in [1, 63, 64, 65, (64 << 10) - 1, (1 << 20) + 1, 5 << 20]:
        s = (np.arange(n, dtype=np.int64) % 251 + rank).astype(np.uint8).view(np.uint8)
        s = s.astype(np.float32)
        r = np.zeros(n, np.float32)
        with comm.group():
            comm.send(s, nxt)
            comm.recv(r, prv)
        assert np.array_equal(r, (np.arange(n, dtype=np.int64) % 251 + prv).astype(np.uint8).astype(np.float32)), n
    # FIFO: three messages to the same peer arrive in order
    outs = [np.zeros(5000, np.int32) for _ in range(3)]
    ins = [np.full(5000, 10 * rank + k, np.int32) for k in range(3)]  # buffers live until group_end
    with comm.group():
        for k in range(3):
            comm.send(ins[k], nxt)
        for k in range(3):
            comm.recv(outs[k], prv)
    for k in range(3):
        assert np.all(outs[k] == 10 * prv + k), "FIFO order"
    # mixed group: collectives and P2P together (10 ops)
    a = np.full(777, rank, np.float64)
    b = np.zeros(777, np.float64)
    mesh_out = [np.zeros(64, np.int64) for _ in range(world)]
    mesh_in = [np.full(64, 100 * rank + q, np.int64) for q in range(world)]
    with comm.group():
        comm.all_reduce(a, out=b)
        for q in range(world):
            if q == rank:
                continue
            comm.send(mesh_in[q], q)
            comm.recv(mesh_out[q], q)
    assert np.all(b == sum(range(world)))
    for q in range(world):
        if q != rank:
            assert np.all(mesh_out[q] == 100 * q + rank), "mesh exchange"
    # Full mesh of 256K int32 (1 MiB) per peer in one group, receives issued in the reverse of
    # the send order (the reference's out-of-order source and mesh cases, test_p2p.cpp:63-78,
    # 264-314).
    big = 1 << 18
    peers = [q for q in range(world) if q != rank]
    big_in = {q: np.arange(big, dtype=np.int32) + 1000 * rank + q for q in peers}
    big_out = {q: np.zeros(big, np.int32) for q in peers}
    with comm.group():
        for q in peers:
            comm.send(big_in[q], q)
        for q in reversed(peers):
            comm.recv(big_out[q], q)
    for q in peers:
        assert np.array_equal(big_out[q], np.arange(big, dtype=np.int32) + 1000 * q + rank), "1 MiB mesh"
    kinds = {q: comm.p2p_transport(q) for q in range(world) if q != rank}
    ex = comm.host_executor
    zc = comm.host_zero_copy
    comm.destroy()
    return {"transports": kinds, "executor": ex, "zero_copy": zc}


def run_init_only(rank: int, world: int) -> Dict:
    """Init and report (used by the bootstrap fault tests; errors propagate as exceptions)."""
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=1, timeout_ms=3000)
    r = comm.rank
    comm.destroy()
    return {"rank": r}


def run_many(rank: int, world: int) -> Dict:
    """all_reduce_many: grouped and ungrouped batches of host tensors, against a local oracle."""
    import torch
    from originccl_b200 import ReduceOp, init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    sizes = [1, 7, 1000, 4096, 70000]
    for grouped in (True, False):
        for op in (ReduceOp.SUM, ReduceOp.MAX, ReduceOp.AVG):
            xs = [torch.from_numpy(value(rank, n, "float32", seed=n + int(op))) for n in sizes]
            batch = comm.batch(xs)
            comm.all_reduce_many(batch, op, scale=1.0, grouped=grouped)
            for n, x in zip(sizes, xs):
                ref = reduce_ref({ReduceOp.SUM: "sum", ReduceOp.MAX: "max", ReduceOp.AVG: "avg"}[op],
                                 [value(r, n, "float32", seed=n + int(op)) for r in range(world)], world)
                assert np.allclose(x.numpy(), ref, rtol=1e-6, atol=1e-6), f"n={n} op={op} grouped={grouped}"
    # out-of-place batch with a fused scale
    xs = [torch.from_numpy(value(rank, n, "float32", seed=5)) for n in sizes]
    outs = [torch.full((n,), 7.0) for n in sizes]
    comm.all_reduce_many(comm.batch(xs, outs), ReduceOp.SUM, scale=0.5)
    for n, o in zip(sizes, outs):
        ref = reduce_ref("sum", [value(r, n, "float32", seed=5) for r in range(world)], world) * 0.5
        assert np.allclose(o.numpy(), ref, rtol=1e-6), f"scaled n={n}"
    comm.destroy()
    return {"ok": True}


def run_abort(rank: int, world: int) -> Dict:
    """Rank 0 starts an AllReduce that rank 1 never joins; another thread aborts the communicator
    after 0.3 s and the call must fail long before the 30 s timeout."""
    import threading
    import time

    from originccl_b200 import BcclError, init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    elapsed = None
    assert comm.async_error() == 0
    if rank == 0:
        x = np.ones(1 << 16, np.float32)
        timer = threading.Timer(0.3, comm.abort)
        timer.start()
        t0 = time.time()
        try:
            comm.all_reduce(x)
            failed = False
        except BcclError:
            failed = True
        elapsed = time.time() - t0
        timer.join()
        assert failed, "aborted AllReduce returned success"
        assert comm.async_error() != 0  # the failure stays visible without another call
    comm.destroy()
    return {"elapsed": elapsed}


_KEEP: List = []


def run_rank_dies(rank: int, world: int) -> Dict:
    """The last rank's process ends 0.5 s after init without finalizing; the others are in an
    AllReduce that needs it and must get an error from the watchdog, long before the 30 s
    timeout."""
    import os
    import threading
    import time

    from originccl_b200 import BcclError, init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    if rank == world - 1:
        _KEEP.append(comm)  # no destroy(): the process just ends
        threading.Timer(0.5, lambda: os._exit(3)).start()
        return {"dies": True}
    x = np.ones(1 << 16, np.float32)
    t0 = time.time()
    try:
        comm.all_reduce(x)
        failed = False
    except BcclError:
        failed = True
    elapsed = time.time() - t0
    assert failed, "AllReduce with a dead peer returned success"
    return {"elapsed": elapsed}


def run_without_shm(rank: int, world: int, part: str) -> Dict:
    """BCCL_DISABLE_SHM=1: the collective matrix ("matrix") or the P2P cases ("p2p") with every
    exchange over TCP, while the communicator still reports one machine."""
    import os
    os.environ["BCCL_DISABLE_SHM"] = "1"
    if part == "matrix":
        return run_matrix(rank, world, [5, 40000], ["float32", "int64"])
    return run_p2p(rank, world)


def run_trace(rank: int, world: int, out_dir: str) -> Dict:
    """BCCL_TRACE on a host communicator: every collective's channel phases become Chrome-trace
    duration events (one track per channel) in the file dump_trace writes."""
    import json
    import os
    os.environ["BCCL_TRACE"] = "100000"
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    big = np.ones(1 << 20, np.float32)         # 4 MiB: split over both channels
    out = np.empty_like(big)
    comm.all_reduce(big, out=out)
    g = np.empty(world * 1000, np.int32)
    comm.all_gather(g, np.full(1000, rank, np.int32))
    with comm.group():
        for _ in range(3):
            comm.all_reduce(np.ones(10, np.float64), out=np.empty(10))
    path = os.path.join(out_dir, f"trace_{rank}.json")
    n = comm.dump_trace(path)
    again = comm.dump_trace(path + ".2")        # cleared by the first dump
    comm.destroy()
    with open(path) as f:
        events = json.load(f)["traceEvents"]
    assert n == len(events) > 0 and again == 0
    assert all(e["ph"] == "X" and e["dur"] >= 0 and e["pid"] == rank for e in events)
    return {"names": sorted({e["name"] for e in events}), "tracks": sorted({e["tid"] for e in events}),
            "ops": sorted({e["args"]["op"] for e in events})}


def run_fuzz(rank: int, world: int, seed: int, n_ops: int, logical_machine_size: int = 0) -> Dict:
    """A random sequence of operations that every rank draws from the same seed: collectives of
    every kind, dtype and op, counts from 0 to a few MiB (odd ones included), in place and out of
    place, random roots, alone or in (nested) groups mixed with Send/Recv around the ring. Every
    result is checked against the oracle, with sentinels, and inputs must come back unchanged."""
    from originccl_b200 import ReduceOp, init_from_env
    comm = init_from_env(n_channels=3, logical_machine_size=logical_machine_size, timeout_ms=60000)
    rng = np.random.default_rng(seed)  # identical on every rank
    checks = []                        # deferred until the group that holds the op has run
    keep = []                          # buffers must live until their group has run
    done = 0

    def draw_count():
        return int(rng.choice([0, 1, 3, 17, 1000, 4097, 65537, 300001, 1 << 20]))

    def one(i: int, grouped: bool):
        kind = str(rng.choice(["allreduce", "reduce", "broadcast", "allgather", "reducescatter", "sendrecv"]))
        dtype = str(rng.choice(["float32", "float64", "int32", "int64"]))
        op = str(rng.choice(list(OPS)))
        n = draw_count()
        root = int(rng.integers(0, world))
        inplace = bool(rng.integers(0, 2))
        tag = f"op {i} {kind} {dtype} {op} n={n} root={root} inplace={inplace}"
        ins = [value(r, n, dtype, seed * 1000 + i) for r in range(world)]
        if kind == "allreduce":
            x = ins[rank].copy()
            if inplace:
                comm.all_reduce(x, ReduceOp(OPS[op]))
                checks.append(lambda: _check(np.append(x, SENTINEL).astype(x.dtype), reduce_ref(op, ins, world), n, tag))
            else:
                y = _out(n, dtype)
                comm.all_reduce(x, ReduceOp(OPS[op]), out=y[:n])
                checks.append(lambda: (_check(y, reduce_ref(op, ins, world), n, tag),
                                       np.testing.assert_array_equal(x, ins[rank], err_msg=tag + " input")))
        elif kind == "reduce":
            x = ins[rank].copy()
            y = _out(n, dtype)
            comm.reduce(x, root, ReduceOp(OPS[op]), out=y[:n] if rank == root else None)
            keep.append(x)
            if rank == root:
                checks.append(lambda: _check(y, reduce_ref(op, ins, world), n, tag))
        elif kind == "broadcast":
            y = _out(n, dtype)
            y[:n] = ins[rank] if rank == root else 0
            comm.broadcast(y[:n], root)
            checks.append(lambda: _check(y, ins[root], n, tag))
        elif kind == "allgather":
            g = _out(n * world, dtype)
            x = ins[rank].copy()
            comm.all_gather(g[:n * world], x)
            keep.append(x)
            checks.append(lambda: _check(g, np.concatenate(ins), n * world, tag))
        elif kind == "reducescatter":
            full = [value(r, n * world, dtype, seed * 1000 + i + 7) for r in range(world)]
            x = full[rank].copy()
            y = _out(n, dtype)
            comm.reduce_scatter(y[:n], x, ReduceOp(OPS[op]))
            keep.append(x)
            checks.append(lambda: _check(y, reduce_ref(op, full, world)[rank * n:(rank + 1) * n], n, tag))
        else:
            if world == 1:
                return
            nxt, prv = (rank + 1) % world, (rank - 1) % world
            s = ins[rank].copy()
            r = _out(n, dtype)
            if grouped:
                comm.send(s, nxt)
                comm.recv(r[:n], prv)
            else:
                with comm.group():
                    comm.send(s, nxt)
                    comm.recv(r[:n], prv)
            checks.append(lambda: _check(r, ins[prv], n, tag))
            keep.append(s)

    i = 0
    while i < n_ops:
        mode = int(rng.integers(0, 3))
        if mode == 0:  # alone
            one(i, False)
            i += 1
        else:          # a group of 2-6 ops, nested once when mode == 2
            k = int(rng.integers(2, 7))
            comm.group_start()
            if mode == 2:
                comm.group_start()
            for _ in range(k):
                one(i, True)
                i += 1
            if mode == 2:
                comm.group_end()  # inner: runs nothing
            comm.group_end()
        for c in checks:
            c()
        done += len(checks)
        checks.clear()
        keep.clear()
    comm.destroy()
    return {"checked": done}


def run_bf16_fp16_torch(rank: int, world: int) -> Dict:
    """bf16 and fp16 on the host path, as torch CPU tensors: the reduction widens to fp32 and
    rounds once (round to nearest even), so results equal the fp32 sum rounded to the type.
    Inputs are multiples of 1/8 in [-8, 8) (exact in both types); sums of a few of them too,
    and AVG / scale results are compared against the same rounding of the fp32 value."""
    import torch

    from originccl_b200 import ReduceOp, init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    checked = 0
    for dt in (torch.bfloat16, torch.float16):
        for n in (1, 7, 4097, 300001):
            ins = [torch.from_numpy(value(r, n, "float32", n + 3)) for r in range(world)]
            x = ins[rank].to(dt)
            for op, scale in (("sum", 1.0), ("max", 1.0), ("min", 1.0), ("avg", 1.0), ("sum", 0.25)):
                if dt == torch.float16 and op == "avg":
                    continue
                y = torch.full((n + 1,), 77.0, dtype=dt)
                comm.all_reduce(x, ReduceOp(OPS[op]), out=y[:n], scale=scale)
                ref = torch.from_numpy(reduce_ref(op, [a.numpy() for a in ins], world).astype(np.float32))
                exp = (ref * scale).to(dt)
                assert torch.equal(y[:n], exp), f"{dt} {op} scale={scale} n={n}: {(y[:n] != exp).nonzero()[:3]}"
                assert y[n].item() == 77.0
                checked += 1
    comm.destroy()
    return {"checked": checked}


def run_all_to_all(rank: int, world: int) -> Dict:
    """Communicator.all_to_all: block q of every rank's input lands in block `rank` of rank q's
    output, for empty, odd and multi-MiB blocks, float32 and int64, and a 2-D tensor."""
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    for n, dt in [(0, np.float32), (1, np.float32), (777, np.int64), ((1 << 20) + 3, np.float32)]:
        x = np.concatenate([np.full(n, 1000 * rank + q, dt) for q in range(world)])
        out = np.full(world * n, -1, dt)
        comm.all_to_all(out, x)
        want = np.concatenate([np.full(n, 1000 * q + rank, dt) for q in range(world)])
        assert np.array_equal(out, want), n
    x2 = np.arange(world * 6, dtype=np.int32).reshape(world * 2, 3) + 100 * rank
    o2 = np.zeros_like(x2)
    comm.all_to_all(o2, x2)
    for q in range(world):
        assert np.array_equal(o2.reshape(-1)[q * 6:(q + 1) * 6], np.arange(rank * 6, rank * 6 + 6) + 100 * q)
    try:
        comm.all_to_all(np.zeros(world * 2 + 1, np.float32), np.zeros(world * 2, np.float32))
        raise AssertionError("mismatched output size accepted")
    except ValueError:
        pass
    comm.destroy()
    return {"ok": True}


def run_split(rank: int, world: int) -> Dict:
    """Communicator.split: even and odd ranks form two communicators ranked in reverse order
    (key = -rank); the last rank also tries a negative color in a second split and gets None;
    collectives run in the children and the parent is still usable afterwards."""
    from originccl_b200 import init_from_env
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    child = comm.split(rank % 2, key=-rank)
    members = sorted((r for r in range(world) if r % 2 == rank % 2), reverse=True)
    assert child.world_size == len(members) and child.rank == members.index(rank)
    x = np.full(1000, rank + 1.0, np.float32)
    child.all_reduce(x)
    assert np.all(x == sum(m + 1 for m in members))
    g = np.empty(len(members) * 3, np.int32)
    child.all_gather(g, np.full(3, rank, np.int32))
    assert list(g[::3]) == members  # child rank order follows the key
    solo = comm.split(-1 if rank == world - 1 else 0)
    assert (solo is None) == (rank == world - 1)
    if solo is not None:
        y = np.ones(5, np.float64)
        solo.all_reduce(y)
        assert np.all(y == world - 1)
        solo.destroy()
    z = np.full(7, 1, np.int64)
    comm.all_reduce(z)  # the parent still works
    assert np.all(z == world)
    child.destroy()
    comm.destroy()
    return {"child_rank": members.index(rank), "child_size": len(members)}


def run_mesh(rank: int, world: int, tp: int) -> Dict:
    """parallel.Mesh: TP groups of consecutive ranks, DP groups of equal TP position; an
    AllReduce in each sums exactly its members."""
    from originccl_b200 import init_from_env
    from originccl_b200.parallel import Mesh
    comm = init_from_env(n_channels=2, timeout_ms=30000)
    mesh = Mesh(comm, tp=tp)
    x = np.full(16, rank + 1.0, np.float64)
    mesh.tp.all_reduce(x)
    g0 = (rank // tp) * tp
    assert np.all(x == sum(r + 1 for r in range(g0, g0 + tp)))
    y = np.full(16, rank + 1.0, np.float64)
    mesh.dp.all_reduce(y)
    assert np.all(y == sum(r + 1 for r in range(rank % tp, world, tp)))
    out = {"tp": (mesh.tp.rank, mesh.tp.world_size), "dp": (mesh.dp.rank, mesh.dp.world_size)}
    mesh.destroy()
    comm.destroy()
    return out


def run_algo_overrides(rank: int, world: int) -> Dict:
    """AllGather / ReduceScatter with an explicit algorithm (the host path has one algorithm, so
    the override is accepted and the result stays exact)."""
    import numpy as np

    import originccl_b200 as occl
    from originccl_b200 import Algo, ReduceOp
    comm = occl.init_from_env()
    n = 1000
    x = (np.arange(n, dtype=np.float32) + rank * 0.5)
    for algo in (Algo.AUTO, Algo.ONESHOT, Algo.NVLS):
        out = np.zeros(n * world, np.float32)
        comm.all_gather(out, x, algo=algo)
        want = np.concatenate([np.arange(n, dtype=np.float32) + r * 0.5 for r in range(world)])
        assert (out == want).all(), algo
        big = np.tile(x, world)
        rs = np.zeros(n, np.float32)
        comm.reduce_scatter(rs, big, ReduceOp.SUM, algo=algo)
        exp = sum(np.arange(n, dtype=np.float32) + r * 0.5 for r in range(world))
        assert (rs == exp).all(), algo
    comm.destroy()
    return {"ok": True}
