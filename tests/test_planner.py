"""Planner white-box tests (CPU): validation, cross-rank ordering, P2P rounds, algorithm table.

Parity: the reference's group/planner cases (OriginCCL tests/test_common.cpp:612-774) check the
SortTasks order (collectives first, P2P last by round), overflow rejection and validation.
"""
import ctypes

from originccl_b200 import _native

AR, BC, RED, AG, RS, SEND, RECV = range(7)
F32, F64, I32, I64, BF16, F16 = range(6)


def sort(rank, world, tasks):
    lib = _native.lib()
    n = len(tasks)
    arr = lambda t, i: (ctypes.c_int * n)(*[x[i] for x in t])  # noqa: E731
    order = (ctypes.c_int * n)()
    counts = (ctypes.c_size_t * n)(*[t[1] for t in tasks])
    rc = lib.bcclPlannerSort(rank, world, n, arr(tasks, 0), counts, arr(tasks, 2), arr(tasks, 3), arr(tasks, 4),
                             arr(tasks, 5), order)
    return rc, list(order)


def test_sort_collectives_first_then_p2p_by_round():
    # (func, count, dtype, op, root, peer)
    tasks = [
        (SEND, 10, F32, 0, 0, 1),      # round for rank 0 -> 1 in world 4: 4 - 1 = 3
        (AR, 100, F32, 0, 0, -1),
        (RECV, 10, F32, 0, 0, 3),      # recv from 3: forward = (0-3+4)%4 = 1 -> round 3
        (AG, 50, F32, 0, 0, -1),
        (AR, 10, F32, 0, 0, -1),
        (SEND, 10, F32, 0, 0, 3),      # forward 3 -> round 1
        (BC, 10, F32, 0, 2, -1),
    ]
    rc, order = sort(0, 4, tasks)
    assert rc == 0
    # collectives by (func, bytes): AR(10), AR(100), BC, AG ; then P2P by round, send before recv
    assert order == [4, 1, 6, 3, 5, 0, 2]


def test_sort_is_stable_for_equal_keys():
    tasks = [(AR, 64, F32, 0, 0, -1)] * 5
    rc, order = sort(1, 2, tasks)
    assert rc == 0 and order == [0, 1, 2, 3, 4]


def test_sort_rejects_invalid_peer_and_overflow():
    assert sort(0, 4, [(SEND, 1, F32, 0, 0, 0)])[0] != 0       # self
    assert sort(0, 4, [(RECV, 1, F32, 0, 0, 4)])[0] != 0       # out of range
    assert sort(0, 4, [(AG, 1 << 62, F32, 0, 0, -1)])[0] != 0   # N*count*size overflows


def test_p2p_rounds_match_the_ring_schedule():
    lib = _native.lib()
    world = 5
    for rank in range(world):
        for i in range(1, world):
            # round i: send to (rank - i), receive from (rank + i)
            assert lib.bcclPlannerP2pRound(SEND, rank, (rank - i) % world, world) == i
            assert lib.bcclPlannerP2pRound(RECV, rank, (rank + i) % world, world) == i


def test_validation_rules():
    lib = _native.lib()
    v = lib.bcclPlannerValidate  # (rank, world, func, count, dtype, op, root, peer, has_send, has_recv)
    assert v(0, 4, AR, 0, F32, 0, 0, -1, 0, 0) == 0            # count 0, no buffers
    assert v(0, 4, AR, 8, F32, 0, 0, -1, 0, 1) != 0            # missing send
    assert v(1, 4, RED, 8, F32, 0, 0, -1, 1, 0) == 0           # non-root reduce, null recv
    assert v(0, 4, RED, 8, F32, 0, 0, -1, 1, 0) != 0           # root needs recv
    assert v(0, 4, BC, 8, F32, 0, 4, -1, 1, 1) != 0            # bad root
    assert v(0, 4, AR, 8, 7, 0, 0, -1, 1, 1) != 0              # bad dtype
    assert v(0, 4, AR, 8, BF16, 5, 0, -1, 1, 1) != 0           # bad op
    assert v(0, 4, AG, 8, F16, 0, 0, -1, 1, 1) == 0


def test_algorithm_table():
    lib = _native.lib()
    algo, ctas = ctypes.c_int(), ctypes.c_int()

    def choose(func, nbytes, world, nvls):
        lib.bcclPlannerChoose(func, F32, 0, nbytes, world, int(nvls), 0, ctypes.byref(algo), ctypes.byref(ctas))
        return algo.value, ctas.value

    ONESHOT, TWOSHOT, NVLS = 1, 2, 3
    assert choose(AR, 8, 8, True)[0] == ONESHOT
    assert choose(AR, 1 << 20, 8, True)[0] == ONESHOT
    assert choose(AR, 4 << 20, 8, True)[0] == TWOSHOT
    assert choose(AR, 64 << 20, 8, True)[0] == NVLS
    assert choose(AR, 64 << 20, 8, False)[0] == TWOSHOT       # no multicast -> two-shot
    assert choose(AR, 4 << 20, 2, True)[0] == TWOSHOT         # two ranks: pipelined push
    assert choose(AR, 32 << 20, 2, True)[0] == 4              # two ranks, mid sizes: ring
    assert choose(AR, 16 << 20, 4, True)[0] == TWOSHOT        # four ranks: two-shot up to 16 MiB
    assert choose(AR, 64 << 20, 4, True)[0] == 5              # then the hybrid
    assert choose(AR, 64 << 20, 4, False)[0] == TWOSHOT       # which needs multicast
    assert choose(AR, 2 << 20, 2, True)[0] == ONESHOT         # two ranks: one-shot push up to 2 MiB
    assert choose(AR, 256 << 20, 2, True)[0] == TWOSHOT       # two ranks, large: two-shot
    assert choose(BC, 256 << 20, 2, True)[0] == ONESHOT       # two ranks: no NVLS for Broadcast
    assert choose(BC, 256 << 20, 8, True)[0] == NVLS
    assert choose(AG, 64 << 20, 8, True)[0] == NVLS           # block leaves the GPU once
    assert choose(AG, 64 << 10, 8, True)[0] == ONESHOT
    assert choose(AG, 64 << 20, 8, False)[0] == ONESHOT      # no multicast
    assert choose(AG, 64 << 20, 2, True)[0] == ONESHOT       # two ranks: nothing to save
    assert choose(RS, 64 << 20, 8, True)[0] == NVLS
    assert choose(RS, 256 << 10, 8, True)[0] == ONESHOT
    assert choose(AR, 8, 8, True)[1] == 1


def test_tuning_table_from_sweeps_is_loaded_by_the_planner(tmp_path, monkeypatch):
    from originccl_b200.utils import tune
    recs = []
    for size, t_one, t_two, t_nvls in [(1024, 5.0, 9.0, 12.0), (65536, 8.0, 7.0, 9.0), (1 << 20, 30.0, 20.0, 15.0),
                                        (1 << 24, 300.0, 120.0, 80.0)]:
        for algo, t in (("oneshot", t_one), ("twoshot", t_two), ("nvls", t_nvls)):
            recs.append({"op": "allreduce", "ranks": 4, "bytes": size, "algo": algo, "time_us": t, "check": True})
    recs.append({"op": "allreduce", "ranks": 4, "bytes": 1 << 24, "algo": "oneshot", "time_us": 1.0, "check": False})
    rows = tune.build_table(recs)
    assert [(r[3], r[2]) for r in rows] == [("oneshot", int((1024 * 65536) ** 0.5)),
                                             ("twoshot", int((65536 * (1 << 20)) ** 0.5)),
                                             ("nvls", (1 << 64) - 1)]
    path = tmp_path / "tuning.txt"
    path.write_text(tune.format_table(rows))
    monkeypatch.setenv("BCCL_TUNING_FILE", str(path))
    lib = _native.lib()
    algo, ctas = ctypes.c_int(), ctypes.c_int()

    def choose(nbytes):
        lib.bcclPlannerChoose(AR, F32, 0, nbytes, 4, 1, 0, ctypes.byref(algo), ctypes.byref(ctas))
        return algo.value

    assert [choose(n) for n in (512, 8192, 65536, 1 << 22, 1 << 30)] == [1, 1, 2, 3, 3]


def test_env_report_runs_without_a_gpu():
    from originccl_b200.utils import env_report
    r = env_report.report()
    assert r["python"] and "bccl" in r and "topology" in r


def test_gemm_tile_width_choice(monkeypatch):
    """2-SM GEMM tile width: 256 by default; BCCL_GEMM_BN=auto takes 224-wide tiles where they
    fill the last wave of 74 CTA pairs better (N = 3584: 448 -> 512 tiles, 7 waves either way),
    and keeps 256 where they do not (runs without a GPU: 148 SMs assumed)."""
    from originccl_b200.ops import gemm
    monkeypatch.setenv("BCCL_GEMM_PAIR", "1")
    monkeypatch.delenv("BCCL_GEMM_BN", raising=False)
    assert gemm.kernel_name(8192, 3584) == "pair_256x256"
    monkeypatch.setenv("BCCL_GEMM_BN", "auto")
    assert gemm.kernel_name(8192, 3584) == "pair_256x224"
    assert gemm.kernel_name(16384, 3584) == "pair_256x224"
    assert gemm.kernel_name(8192, 8192) == "pair_256x256"
    assert gemm.kernel_name(4096, 4096) == "pair_256x256"
    monkeypatch.setenv("BCCL_GEMM_BN", "224")
    assert gemm.kernel_name(4096, 4096) == "pair_256x224"
    monkeypatch.setenv("BCCL_GEMM_PAIR", "0")
    assert gemm.kernel_name(8192, 3584) == "single_128x256"
