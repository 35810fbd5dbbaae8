"""pip packaging: a wheel built offline from the source tree carries the native library, and the
installed package (outside the source tree) runs a collective with it."""
import glob
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROBE = r"""
import numpy as np, originccl_b200 as occl, os
assert not occl.__file__.startswith(os.environ["SRC"]), occl.__file__
comm = occl.Communicator().init(0, 1, None)
x = np.arange(8, dtype=np.float32); y = np.empty_like(x)
comm.all_reduce(x, out=y, scale=2.0)
assert np.array_equal(y, 2 * x)
comm.destroy()
print("installed ok", occl.version())
"""


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    assert r.returncode == 0, " ".join(cmd) + "\n" + (r.stdout + r.stderr)[-4000:]
    return r


def test_wheel_builds_and_installed_package_runs(tmp_path):
    wheels, target = tmp_path / "wheels", tmp_path / "site"
    _run([sys.executable, "-m", "pip", "wheel", "--no-build-isolation", "--no-deps", "--no-index", "-w", str(wheels),
          ROOT], timeout=1500)
    whl = glob.glob(str(wheels / "originccl_b200-*.whl"))
    assert len(whl) == 1 and "none-any" not in whl[0], whl  # platform wheel: it carries libbccl.so
    _run([sys.executable, "-m", "pip", "install", "--no-deps", "--no-index", "--target", str(target), whl[0]],
         timeout=300)
    assert (target / "originccl_b200" / "_lib" / "libbccl.so").exists()
    env = dict(os.environ, PYTHONPATH=str(target), SRC=ROOT)
    r = _run([sys.executable, "-c", PROBE], timeout=120, cwd=str(tmp_path), env=env)
    assert "installed ok" in r.stdout
