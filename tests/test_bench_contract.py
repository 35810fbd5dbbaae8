"""The benchmark entry points' contract, on CPU: `bench.py --impl reference` prints one JSON line
(the reference has no GPU path and cannot be built here, so the line says why) and exits 0, also
when launched by torchrun on several ranks as the scaling run does; a GPU count that disagrees
with the launcher is refused; `__graft_entry__.build` compiles and imports the package."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _json_lines(text):
    return [json.loads(l) for l in text.splitlines() if l.startswith("{")]


def test_reference_arm_one_rank():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=ROOT, capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = _json_lines(r.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["unavailable"]


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29561", "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference"


def test_gpu_count_must_match_the_launcher():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    r = subprocess.run([sys.executable, "bench.py", "--gpus", "2"], cwd=ROOT, capture_output=True, text=True,
                       timeout=120, env=env)
    assert r.returncode != 0 and "WORLD_SIZE" in (r.stdout + r.stderr)


def test_graft_entry_build_imports_the_package():
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.build(); "
                        "import originccl_b200; print(originccl_b200.version())"],
                       cwd=ROOT, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip()
