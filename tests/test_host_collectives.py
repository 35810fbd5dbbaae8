"""Host-memory communicator (CPU ranks over shared memory and TCP) -- no GPU needed."""
import pytest

from tests import _mp, host_cases


def test_level0_matrix_four_ranks_one_machine():
    res = _mp.run(4, host_cases.run_matrix, [1, 128, 32768, 131072 + 3], ["float32", "int32"], timeout=300)
    assert all(r["ran"] > 0 for r in res)
    assert res[0]["single"] and res[0]["local_size"] == 4 and res[0]["local_ranks"] == [0, 1, 2, 3]


def test_all_dtypes_odd_sizes():
    res = _mp.run(3, host_cases.run_matrix, [7, 4099], ["float32", "float64", "int32", "int64", "float16"], 3,
                  timeout=300)
    assert res[0]["ran"] > 0


def test_logical_two_machines():
    # Ranks r and s share a logical machine iff r // 2 == s // 2 (hostname injection).
    res = _mp.run(4, host_cases.run_matrix, [1000, 70001], ["float32", "int64"], 2, 2, timeout=300)
    assert res[0]["machine_count"] == 2 and res[0]["leaders"] == [0, 2]
    assert res[3]["local_ranks"] == [2, 3] and res[3]["machine_index"] == 1 and res[3]["local_rank"] == 1
    assert not res[0]["single"]


def test_logical_uneven_machines():
    res = _mp.run(5, host_cases.run_matrix, [513], ["float64"], 1, 2, timeout=300)
    assert res[0]["machine_count"] == 3 and res[4]["local_ranks"] == [4] and res[0]["leaders"] == [0, 2, 4]


def test_contract_cases():
    res = _mp.run(3, host_cases.run_contract, timeout=120)
    assert res[0]["rejected"] == 9


def test_nested_groups():
    res = _mp.run(3, host_cases.run_groups, timeout=120)
    assert all(r["inner_untouched"] for r in res)


def test_single_rank():
    res = _mp.run(1, host_cases.run_matrix, [5, 1000], ["float32", "int32"], timeout=120)
    assert res[0]["ran"] > 0


def test_p2p_shared_memory():
    res = _mp.run(4, host_cases.run_p2p, timeout=300)
    assert set(res[0]["transports"].values()) == {"shm"}
    # Messages of 256 KiB and more went single-copy (process_vm_readv) where the host allows it.
    enabled, received = res[0]["zero_copy"]
    assert not enabled or received == 5  # 2 ring messages of 4 and 20 MiB + three 1 MiB mesh messages


def test_p2p_shared_memory_without_zero_copy():
    res = _mp.run(3, host_cases.run_p2p, 0, "", "0", timeout=300)
    assert all(r["zero_copy"] == (False, 0) for r in res)


def test_p2p_across_logical_machines_tcp_epoll():
    res = _mp.run(4, host_cases.run_p2p, 2, "epoll", timeout=300)
    assert res[0]["transports"] == {1: "shm", 2: "tcp", 3: "tcp"}
    assert res[0]["executor"] == "epoll"


def test_all_reduce_many_batches():
    res = _mp.run(3, host_cases.run_many, timeout=240)
    assert all(r["ok"] for r in res)


def test_four_logical_machines_leader_ring():
    # Four machines of one rank each: AllReduce between machines runs the leaders' ring.
    res = _mp.run(4, host_cases.run_matrix, [1, 5, 4099, 70001], ["float32", "int32", "float64"], 2, 1,
                  timeout=300)
    assert res[0]["machine_count"] == 4 and res[0]["leaders"] == [0, 1, 2, 3]


def test_three_logical_machines_of_two_ranks():
    res = _mp.run(6, host_cases.run_matrix, [3, 1000, 131072 + 7], ["float32", "int64"], 2, 2, timeout=400)
    assert res[0]["machine_count"] == 3 and res[5]["local_ranks"] == [4, 5]


def test_disable_shm_runs_everything_over_tcp():
    res = _mp.run(4, host_cases.run_without_shm, "matrix", timeout=300)
    assert res[0]["ran"] > 0 and res[0]["single"]  # the view stays one machine
    res = _mp.run(4, host_cases.run_without_shm, "p2p", timeout=300)
    assert set(res[0]["transports"].values()) == {"tcp"}


def test_host_trace_records_channel_phases(tmp_path):
    res = _mp.run(2, host_cases.run_trace, str(tmp_path), timeout=120)
    for r in res:
        assert {"copy_in", "barrier_wait", "reduce", "copy_out"} <= set(r["names"])
        assert r["tracks"] == [0, 1] and {"allreduce", "allgather"} <= set(r["ops"])


@pytest.mark.parametrize("world,machine,seed", [(3, 0, 11), (4, 2, 12), (5, 2, 13)])
def test_random_operation_sequences(world, machine, seed):
    res = _mp.run(world, host_cases.run_fuzz, seed, 120, machine, timeout=600)
    assert all(r["checked"] >= 60 for r in res)


def test_bf16_fp16_on_host_tensors():
    res = _mp.run(3, host_cases.run_bf16_fp16_torch, timeout=180)
    assert all(r["checked"] == 36 for r in res)


@pytest.mark.parametrize("world", [1, 3, 4])
def test_all_to_all(world):
    _mp.run(world, host_cases.run_all_to_all, timeout=180)


def test_communicator_split():
    res = _mp.run(5, host_cases.run_split, timeout=180)
    assert [r["child_rank"] for r in res] == [2, 1, 1, 0, 0] and [r["child_size"] for r in res] == [3, 2, 3, 2, 3]


def test_tp_dp_mesh():
    res = _mp.run(6, host_cases.run_mesh, 3, timeout=180)
    assert [r["tp"] for r in res] == [(0, 3), (1, 3), (2, 3)] * 2
    assert [r["dp"] for r in res] == [(0, 2)] * 3 + [(1, 2)] * 3


def test_several_single_rank_communicators_in_one_process():
    # One-rank communicators share no unique id; each still needs its own local socket name.
    import numpy as np

    import originccl_b200 as occl
    comms = [occl.Communicator().init(0, 1, None) for _ in range(3)]
    x = np.arange(8, dtype=np.float32)
    for c in comms:
        c.all_reduce(x)
    assert (x == np.arange(8, dtype=np.float32)).all()
    for c in comms:
        c.destroy()


def test_allgather_reducescatter_algorithm_override():
    res = _mp.run(3, host_cases.run_algo_overrides, timeout=120)
    assert all(r["ok"] for r in res)
