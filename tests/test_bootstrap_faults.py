"""Failure detection on the host (CPU ranks only; nothing here touches a GPU).

Faults are injected with BCCL_FAULT in the failing rank; every rank must come back with an
error within the bootstrap timeout instead of hanging. Parity: the reference bounds its
bootstrap connect/retry (OriginCCL src/bootstrap.cpp:71, src/utils.cpp:128-138) but has no
fault injection; these cases exercise the bounded paths.
"""
import os
import time

from tests import _mp, host_cases

ENV = {"BCCL_BOOTSTRAP_TIMEOUT_MS": "3000"}


def _run_with_fault(world, fault):
    env = dict(ENV, BCCL_FAULT=fault)
    t0 = time.time()
    res = _mp.run(world, host_cases.run_init_only, timeout=60, env=env, expect_fail=True)
    return res, time.time() - t0


def test_rank_that_never_joins():
    res, dt = _run_with_fault(3, "bootstrap_skip:2")
    assert all(not ok for ok, _ in res), res
    assert dt < 30


def test_corrupted_hello_is_rejected():
    res, _ = _run_with_fault(3, "bootstrap_corrupt:1")
    assert not res[0][0] and not res[1][0]


def test_late_rank_within_timeout_is_fine():
    res, _ = _run_with_fault(3, "bootstrap_delay:1:500")
    assert all(ok for ok, _ in res), res


def test_shared_segment_never_arrives():
    res, dt = _run_with_fault(3, "segment_drop:0")
    assert not any(ok for ok, _ in res[1:]), res
    assert dt < 30


def test_abort_stops_a_collective_a_peer_never_joins():
    res = _mp.run(2, host_cases.run_abort, timeout=120)
    assert res[0]["elapsed"] < 5.0


def test_watchdog_reports_a_rank_that_dies():
    res = _mp.run(3, host_cases.run_rank_dies, timeout=120)
    assert res[2]["dies"]
    assert res[0]["elapsed"] < 10.0 and res[1]["elapsed"] < 10.0, res
