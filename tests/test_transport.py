"""Host transport semantics (TCP socket and shared-memory ring): the suite in
csrc/examples/bccl_transport_check.cc, run as two processes per transport."""
import json
import os
import subprocess

import pytest

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "originccl_b200", "_lib")
BIN = os.path.join(LIB, "bccl_transport_check")


@pytest.mark.parametrize("transport", ["tcp", "shm"])
def test_transport_semantics(transport):
    if not os.path.exists(BIN):
        from originccl_b200 import _build
        _build.build()
    r = subprocess.run([BIN, transport], capture_output=True, text=True, timeout=120)
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    assert r.returncode == 0 and lines, r.stdout + r.stderr
    res = lines[-1]
    assert res["transport"] == transport and res["failed"] == 0 and res["passed"] >= 25, res
