"""The host path under AddressSanitizer + UndefinedBehaviorSanitizer and under ThreadSanitizer.

The library's host C++ (communicator, bootstrap, planner, host engine with its channel threads,
transports, watchdog) and the example programs are rebuilt with ``-fsanitize=...``
(``originccl_b200._build.build_sanitized``) and the C++ check matrix, the benchmarks and the
transport suite run under them as several processes. Any report fails the test: UBSan and TSan
halt on the first one, ASan on its first error and LeakSanitizer at exit. The reference has no
sanitizer build (it suggests configuring one by hand); CUDA kernels are not instrumented and
compute-sanitizer is not used.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUN = os.path.join(ROOT, "originccl_b200", "_lib", "bccl_run")

ENV = {
    "ASAN_OPTIONS": "detect_leaks=1:halt_on_error=1:detect_stack_use_after_return=1",
    "UBSAN_OPTIONS": "halt_on_error=1:print_stacktrace=1",
    "TSAN_OPTIONS": "halt_on_error=1:second_deadlock_stack=1",
}
REPORTS = ("ERROR: AddressSanitizer", "ERROR: LeakSanitizer", "runtime error:", "WARNING: ThreadSanitizer")

CASES = [
    ["-np", "4", "--", "{bin}/bccl_check", "check"],
    ["-np", "6", "--", "{bin}/bccl_check", "check", "--ranks-per-machine", "2"],
    ["-np", "4", "--", "{bin}/bccl_check", "bench", "--counts", "1000,300000,3000000", "--warmup", "2", "--iters", "5"],
    ["-np", "4", "--", "{bin}/bccl_check", "bench-group", "--messages", "64", "--message-bytes", "65536", "--warmup",
     "2", "--iters", "5"],
    ["-np", "4", "--", "{bin}/bccl_check", "fuzz", "--seed", "7", "--ops", "40"],
    ["-np", "6", "--", "{bin}/bccl_check", "fuzz", "--seed", "8", "--ops", "30", "--ranks-per-machine", "2"],
]


@pytest.fixture(scope="module", params=["asan", "tsan"])
def sanitized(request):
    from originccl_b200 import _build
    return request.param, str(_build.build_sanitized(request.param))


def _check(r):
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-6000:]
    assert not [line for line in out.splitlines() if any(k in line for k in REPORTS)], out[-6000:]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_host_collectives_under_sanitizer(sanitized, case):
    kind, bin_dir = sanitized
    args = [a.format(bin=bin_dir) for a in CASES[case]]
    env = dict(os.environ, **ENV)
    r = subprocess.run([RUN, "--timeout", "240"] + args, capture_output=True, text=True, timeout=300, env=env)
    _check(r)


@pytest.mark.parametrize("transport", ["tcp", "shm"])
def test_transport_suite_under_sanitizer(sanitized, transport):
    kind, bin_dir = sanitized
    env = dict(os.environ, **ENV)
    r = subprocess.run([os.path.join(bin_dir, "bccl_transport_check"), transport], capture_output=True, text=True,
                       timeout=240, env=env)
    _check(r)
    assert '"failed": 0' in r.stdout
