"""The C++ API end to end: the bccl_run launcher starting ranks of the bccl_check program
(csrc/examples/bccl_check.cc), which uses bccl::Communicator directly (no Python in the ranks)."""
import json
import os
import subprocess
import time

import pytest

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "originccl_b200", "_lib")
RUN = os.path.join(LIB, "bccl_run")
CHECK = os.path.join(LIB, "bccl_check")


def _need_binaries():
    if not (os.path.exists(RUN) and os.path.exists(CHECK)):
        from originccl_b200 import _build
        _build.build()


def _run(args, timeout=180):
    _need_binaries()
    return subprocess.run([RUN] + args, capture_output=True, text=True, timeout=timeout)


def _json_lines(out):
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


# The reference's levels run 4, 8 and 32 ranks (tests/test_common.cpp:28-39); its multi-machine
# test groups ranks into logical machines by hostname (tests/regression/test_multi_machine.cpp).
@pytest.mark.parametrize("np_,per_machine,machines", [
    (1, 0, 1), (2, 0, 1), (4, 0, 1),    # one machine, level 0
    (8, 0, 1),                          # level 1
    (32, 8, 4),                         # level 2: four logical machines of eight ranks
    (8, 3, 3),                          # uneven machines (3 + 3 + 2)
    (4, 1, 4),                          # one rank per machine: every exchange over TCP
])
def test_cpp_check_matrix_host(np_, per_machine, machines):
    extra = ["--ranks-per-machine", str(per_machine)] if per_machine else []
    r = _run(["-np", str(np_), "--timeout", "150", "--", CHECK, "check"] + extra)
    assert r.returncode == 0, r.stdout + r.stderr
    res = _json_lines(r.stdout)[-1]
    assert res["failed_all_ranks"] == 0 and res["passed"] >= 56 and res["ranks"] == np_
    assert res["machines"] == machines


def test_cpp_int32_allreduce_bench_host():
    r = _run(["-np", "4", "--timeout", "150", "--", CHECK, "bench", "--counts", "32768,131072", "--warmup", "3",
              "--iters", "10"])
    assert r.returncode == 0, r.stdout + r.stderr
    recs = _json_lines(r.stdout)
    assert [x["count"] for x in recs] == [32768, 131072]
    assert all(x["check"] and x["busbw_gbs"] > 0 for x in recs)


def test_launcher_stops_all_ranks_when_one_fails():
    t0 = time.time()
    r = _run(["-np", "3", "--", "sh", "-c", 'if [ "$BCCL_RANK" = 1 ]; then exit 7; fi; sleep 60'], timeout=60)
    assert r.returncode == 7
    assert time.time() - t0 < 30
    assert "rank 1 exited with 7" in r.stderr


def test_launcher_exports_rank_environment():
    r = _run(["-np", "2", "--", "sh", "-c", 'echo "$BCCL_RANK/$BCCL_WORLD_SIZE/$BCCL_LOCAL_RANK ${BCCL_ID_FILE:+id}"'])
    assert r.returncode == 0
    assert sorted(r.stdout.split("\n")[:2]) == ["0/2/0 id", "1/2/1 id"]


def test_launcher_timeout():
    r = _run(["-np", "2", "--timeout", "1", "--", "sleep", "30"], timeout=60)
    assert r.returncode == 124


@pytest.mark.gpu
def test_cpp_check_matrix_device_one_gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    r = _run(["-np", "1", "--gpus", "--timeout", "150", "--", CHECK, "check", "--device"])
    assert r.returncode == 0, r.stdout + r.stderr
    res = _json_lines(r.stdout)[-1]
    assert res["failed_all_ranks"] == 0 and res["path"] == "device"


def test_cpp_group_benchmark_host_many_small_messages():
    # The reference's --group-small case: many 256 KiB AllReduces in one group, spread over the
    # channel threads by the host engine's planner.
    r = _run(["-np", "3", "--timeout", "150", "--", CHECK, "bench-group", "--messages", "24",
              "--message-bytes", "65536", "--warmup", "2", "--iters", "3"])
    assert r.returncode == 0, r.stdout + r.stderr
    rec = _json_lines(r.stdout)[-1]
    assert rec["check"] and rec["messages"] == 24 and rec["msgs_per_s"] > 0


def test_python_launcher_runs_python_ranks():
    import sys
    code = ("import sys; sys.path.insert(0, %r); import numpy as np, originccl_b200 as o; c = o.init_from_env(); "
            "x = np.full(4, c.rank + 1.0, np.float32); c.all_reduce(x); assert (x == 3).all(); c.destroy()"
            % os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    r = subprocess.run([sys.executable, "-m", "originccl_b200.run", "-np", "2", "--timeout", "60", "--",
                        sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stdout + r.stderr


def _free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("program", ["cpp", "python"])
def test_multi_node_launch(program):
    """Two launcher instances ("nodes") started like torchrun: --nnodes 2 --node-rank K --master
    ADDR:PORT; no id file, rank 0 listens on the master port. The ranks group into two logical
    machines (hostname injection), so the collectives cross them over TCP."""
    import sys
    _need_binaries()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    port = _free_port()
    if program == "cpp":
        prog = [CHECK, "check", "--ranks-per-machine", "2"]
    else:
        code = ("import sys; sys.path.insert(0, %r); import numpy as np, originccl_b200 as o; "
                "c = o.init_from_env(logical_machine_size=2); x = np.full(4, c.rank + 1.0, np.float32); "
                "c.all_reduce(x); assert (x == 10).all(), x; assert c.machine_count == 2; "
                "import os; os.write(1, ('rank %%d of %%d\\n' %% (c.rank, c.world_size)).encode()); c.destroy()"
                % root)
        prog = [sys.executable, "-c", code]
    procs = [subprocess.Popen([RUN, "-np", "2", "--nnodes", "2", "--node-rank", str(k), "--master",
                               f"127.0.0.1:{port}", "--timeout", "120", "--"] + prog,
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, cwd=root)
             for k in (0, 1)]
    outs = [p.communicate(timeout=180) for p in procs]
    for p, (out, err) in zip(procs, outs):
        assert p.returncode == 0, out + err
    if program == "cpp":
        res = _json_lines(outs[0][0])[-1]
        assert res["failed_all_ranks"] == 0 and res["ranks"] == 4 and res["machines"] == 2
    else:
        assert sorted(l for o, _ in outs for l in o.splitlines() if l.startswith("rank")) == \
            [f"rank {r} of 4" for r in range(4)]


@pytest.mark.parametrize("np_", [1, 3])
def test_c_interface_from_c11(np_):
    """csrc/examples/bccl_c_example.c: the C header compiled as C11 (-pedantic) and the library
    driven from plain C: AllReduce, a grouped AllGather + ReduceScatter, Send/Recv."""
    prog = os.path.join(LIB, "bccl_c_example")
    if not os.path.exists(prog):
        from originccl_b200 import _build
        _build.build()
    r = _run(["-np", str(np_), "--timeout", "60", "--", prog])
    assert r.returncode == 0, r.stdout + r.stderr
    assert sorted(l for l in r.stdout.splitlines() if l.startswith("rank")) == \
        sorted(f"rank {q} of {np_}: ok" for q in range(np_))


@pytest.mark.parametrize("args", [
    ["--op", "allreduce", "--dtype", "bf16", "--redop", "avg"],
    ["--op", "allgather", "--dtype", "f16"],
    ["--op", "reducescatter", "--dtype", "i32", "--redop", "max"],
    ["--op", "broadcast", "--dtype", "f64", "--root", "2", "--inplace"],
    ["--op", "reduce", "--dtype", "i64", "--redop", "min", "--root", "1"],
    ["--op", "sendrecv", "--dtype", "f32"],
])
def test_perf_tool_host(args):
    """bccl_perf (the reference's size-sweep benchmark for every collective) on host buffers:
    every size is validated before it is timed and reported as a JSON line."""
    perf = os.path.join(LIB, "bccl_perf")
    if not os.path.exists(perf):
        from originccl_b200 import _build
        _build.build()
    r = _run(["-np", "3", "--timeout", "120", "--", perf, "-b", "4", "-e", "2M", "-f", "8", "-w", "1", "-n", "3",
              "--json"] + args)
    assert r.returncode == 0, r.stdout + r.stderr
    recs = _json_lines(r.stdout)
    assert len(recs) >= 6 and all(x["check"] and x["time_us"] > 0 and x["ranks"] == 3 for x in recs)


@pytest.mark.gpu
@pytest.mark.parametrize("op", ["allreduce", "allgather", "reducescatter", "broadcast", "reduce"])
def test_perf_tool_device_one_gpu(op):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    r = _run(["-np", "1", "--gpus", "--timeout", "120", "--", os.path.join(LIB, "bccl_perf"), "--device", "--op", op,
              "--dtype", "bf16", "-b", "4", "-e", "64M", "-f", "16", "-w", "2", "-n", "5", "--json"])
    assert r.returncode == 0, r.stdout + r.stderr
    recs = _json_lines(r.stdout)
    assert len(recs) >= 6 and all(x["check"] and x["path"] == "device" for x in recs)


def test_launcher_tag_output():
    r = _run(["-np", "3", "--tag-output", "--", "sh", "-c",
              'echo out $BCCL_RANK; echo err $BCCL_RANK >&2; printf "tail $BCCL_RANK"'])
    assert r.returncode == 0
    out = sorted(r.stdout.splitlines())
    assert out == sorted([f"[rank {q}] out {q}" for q in range(3)] + [f"[rank {q}] tail {q}" for q in range(3)])
    assert sorted(r.stderr.splitlines()) == [f"[rank {q}] err {q}" for q in range(3)]
