"""Device communicator tests (need a B200). Numerics are checked against a float64 host oracle."""

import pytest

torch = pytest.importorskip("torch")

from tests import _mp, gpu_cases  # noqa: E402

pytestmark = pytest.mark.gpu


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPU(s)")


def test_native_library_is_the_in_tree_build():
    _need(1)
    from originccl_b200 import _native
    lib = _native.lib()
    assert str(_native._LIB_PATH) == lib._name


def test_single_rank_suite():
    _need(1)
    res = _mp.run(1, gpu_cases.run_suite, [1, 7, 4097, (1 << 20) + 3], ["auto"], timeout=600)
    assert res[0]["ran"] > 0
    assert res[0]["group_launches"] == 1  # 64 collectives in one group -> one batched kernel


def test_single_rank_large_multi_round():
    _need(1)
    # Larger than the per-round staging slot: several rounds in one launch.
    res = _mp.run(1, gpu_cases.run_suite, [(96 << 20) // 4 + 5], ["auto"], True, timeout=600)
    assert res[0]["ran"] > 0


@pytest.mark.multigpu
def test_two_rank_suite_all_algorithms():
    _need(2)
    res = _mp.run(2, gpu_cases.run_suite, [1, 33, 4099, 65537, (3 << 20) + 5],
                  ["oneshot", "twoshot", "nvls", "ring", "hybrid", "ll", "auto"], timeout=900)
    assert "ring" in res[0]["algorithms"] and "ll" in res[0]["algorithms"]
    assert "hybrid" in res[0]["algorithms"] or not res[0]["nvls"]
    assert "rs:nvls" in res[0]["algorithms"] or not res[0]["nvls"]
    assert res[0]["ran"] > 0


# Small staging buffers: every kernel runs many rounds and reuses its staging slots within one
# launch, with a shorter last round (the case where CTA ranges must stay fixed across rounds).
_SMALL_STAGING = {"BCCL_BUFFSIZE": str(16 << 20), "BCCL_NVLS_BUFFSIZE": str(16 << 20),
                  "BCCL_PIPE_MIN_CHUNK": str(64 << 10)}


@pytest.mark.multigpu
def test_two_rank_many_rounds_reusing_slots():
    # Device counters are compared across ranks after every call.
    _need(2)
    res = _mp.run(2, gpu_cases.run_suite, [(9 << 20) + 7], ["twoshot", "nvls", "hybrid", "ring", "auto"], True,
                  timeout=900, env=_SMALL_STAGING)
    assert res[0]["ran"] > 0


@pytest.mark.multigpu
def test_two_rank_pipelines_with_barrier_lag():
    # BCCL_PIPE_LAG=2: iteration t waits for barrier t-2 over a five-slot ring; many rounds.
    _need(2)
    res = _mp.run(2, gpu_cases.run_suite, [(3 << 20) + 5, (9 << 20) + 7], ["twoshot", "nvls", "hybrid", "auto"],
                  True, timeout=900, env={**_SMALL_STAGING, "BCCL_PIPE_LAG": "2"})
    assert res[0]["ran"] > 0


@pytest.mark.multigpu
def test_all_gpu_suite():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 3:
        pytest.skip("needs 3+ GPUs")
    n = min(n, 8)
    res = _mp.run(n, gpu_cases.run_suite, [5, 3001, 70001, (9 << 20) + 7], ["oneshot", "twoshot", "nvls", "hybrid", "ll"],
                  True, timeout=900)
    assert res[0]["ran"] > 0


@pytest.mark.multigpu
def test_all_gpu_many_rounds_reusing_slots():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 3:
        pytest.skip("needs 3+ GPUs")
    for lag in ("1", "2"):
        res = _mp.run(min(n, 8), gpu_cases.run_suite, [(3 << 20) + 7], ["twoshot", "nvls", "hybrid", "auto"], True,
                      timeout=900, env={**_SMALL_STAGING, "BCCL_BUFFSIZE": str(8 << 20), "BCCL_PIPE_LAG": lag})
        assert res[0]["ran"] > 0


@pytest.mark.multigpu
def test_p2p_ring_over_nccl():
    _need(2)
    _mp.run(2, gpu_cases.run_p2p, timeout=300)


@pytest.mark.multigpu
def test_p2p_native_kernel():
    n = min(torch.cuda.device_count(), 4) if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2 GPUs")
    res = _mp.run(n, gpu_cases.run_p2p_native, timeout=300, env={"BCCL_P2P_NATIVE": "1"})
    assert res[0]["algorithms"] == ["native_p2p"]


@pytest.mark.multigpu
def test_bounded_wait_reports_timeout():
    _need(2)
    res = _mp.run(2, gpu_cases.run_timeout_probe, timeout=300, env={"NCCL_NVLS_ENABLE": "0"})
    assert res[0]["raised"], res[0]
    assert "timeout" in res[0]["msg"], res[0]
    assert res[0]["context_ok"]


def test_bounded_wait_self_test_single_gpu():
    """A kernel waiting on a flag nothing sets gives up after ~0.2 s and reports a timeout."""
    _need(1)
    import time
    import originccl_b200 as occl
    from originccl_b200 import _native
    torch.cuda.set_device(0)
    comm = occl.Communicator().init(0, 1, None, device=0, blocking=True)
    t0 = time.time()
    code = _native.lib().bcclDebugWaitProbe(comm._h, 200)
    assert code == 1, code
    assert time.time() - t0 < 10
    # The context and the communicator still work afterwards.
    x = torch.ones(1000, device="cuda")
    comm.all_reduce(x, scale=3.0)
    assert torch.all(x == 3.0).item()
    comm.destroy()


@pytest.mark.multigpu
def test_mixed_algorithm_sequence():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2+ GPUs")
    res = _mp.run(min(n, 8), gpu_cases.run_mixed_sequence, timeout=900)
    assert res[0]["checked"] > 0


def test_tp_fused_single_rank():
    _need(1)
    res = _mp.run(1, gpu_cases.run_tp, timeout=300)
    assert res[0]["ag_err"] < 2e-2


@pytest.mark.multigpu
@pytest.mark.parametrize("multicast", ["0", "1"])
def test_tp_fused_two_ranks(multicast):
    # Both pushes of the gathered chunks: per-peer stores (default) and multimem.st (opt-in).
    _need(2)
    res = _mp.run(2, gpu_cases.run_tp, timeout=600, env={"BCCL_TP_MULTICAST": multicast})
    assert res[0]["ag_err"] < 2e-2 and res[0]["rs_err"] < 3e-2


@pytest.mark.multigpu
def test_tp_fused_all_gpus():
    # TP = every GPU (8 on an HGX box): GEMM->ReduceScatter sums bf16 partial tiles of all ranks in
    # fp32; checked against an fp32 PyTorch reference of the whole MLP block.
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 3:
        pytest.skip("needs 3+ GPUs")
    res = _mp.run(min(n, 8), gpu_cases.run_tp, timeout=900)
    assert res[0]["ag_err"] < 2e-2 and res[0]["rs_err"] < 3e-2


@pytest.mark.multigpu
def test_data_parallel_sync_two_ranks():
    _need(2)
    res = _mp.run(2, gpu_cases.run_dp, timeout=300)
    # cudaMalloc'd gradient storage: registered by default, buckets reduced over peer memory.
    assert res[0]["buckets"] > 1 and res[0]["small"] > 0 and res[0]["registered"]


@pytest.mark.multigpu
def test_zero_copy_nvls_two_ranks():
    _need(2)
    res = _mp.run(2, gpu_cases.run_zero_copy, timeout=300)
    # The large cases run the zero-copy NVLS kernel; the smallest AllGather (4 KiB blocks) takes
    # the low-latency kernel, which the planner prefers for small ungrouped blocks on any buffer.
    assert res[0].get("skipped") or ("nvls_zero_copy" in res[0]["algorithms"] and
                                     set(res[0]["algorithms"]) <= {"nvls_zero_copy", "ll"})


def test_cuda_graph_replay_single_rank():
    _need(1)
    res = _mp.run(1, gpu_cases.run_graph, timeout=300)
    assert res[0]["replays"] == 4 and res[0]["host_launches_during_replays"] == 0


@pytest.mark.multigpu
def test_cuda_graph_replay_two_ranks():
    _need(2)
    res = _mp.run(2, gpu_cases.run_graph, timeout=300)
    assert all(r["host_launches_during_replays"] == 0 for r in res)


@pytest.mark.multigpu
def test_registered_buffers_zero_copy_two_ranks():
    _need(2)
    res = _mp.run(2, gpu_cases.run_registered, timeout=300)
    assert res[0]["algorithms"] == ["p2p_zero_copy"] and res[0]["small_algorithm"] in ("oneshot", "ll")


@pytest.mark.parametrize("world", [1, 2])
def test_random_device_operation_sequences(world):
    _need(world)
    res = _mp.run(world, gpu_cases.run_fuzz, 5 + world, 60, timeout=600)
    assert all(r["checked"] >= 30 for r in res)


@pytest.mark.multigpu
def test_split_device_communicators():
    _need(2)
    res = _mp.run(2, gpu_cases.run_split_device, timeout=300)
    assert [r["both_rank"] for r in res] == [1, 0] and all(r["alone_size"] == 1 for r in res)
