"""The CMake build (the reference's build system) end to end: configure and build the library,
the launcher and the example programs with CMake, run the C++ check matrix with the CMake-built
binaries, install, and build and run a separate consumer project that uses
``find_package(bccl)`` and links ``bccl::bccl``. Kernels are cross-compiled for sm_100a; the
programs run on host memory, so no GPU is needed."""
import json
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NVCC = "/usr/local/cuda/bin/nvcc"

CONSUMER_CMAKE = """
cmake_minimum_required(VERSION 3.24)
project(bccl_consumer LANGUAGES CXX)
find_package(bccl REQUIRED)
add_executable(consumer main.cc)
target_link_libraries(consumer PRIVATE bccl::bccl)
"""

CONSUMER_MAIN = r"""
#include <cstdio>
#include "bccl/communicator.h"

int main() {
    bccl::Communicator comm;
    bccl::CommConfig cfg;
    cfg.rank = 0;
    cfg.world_size = 1;
    if (!comm.GetUniqueId(cfg.unique_id) || !comm.Init(cfg)) return 2;
    int x[4] = {1, 2, 3, 4}, y[4] = {0, 0, 0, 0};
    if (!comm.AllReduce(x, y, 4, bccl::DataType::INT32, bccl::ReduceOp::SUM)) return 3;
    comm.Finalize();
    std::printf("consumer %d %d %d %d\n", y[0], y[1], y[2], y[3]);
    return (y[0] == 1 && y[3] == 4) ? 0 : 4;
}
"""


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    assert r.returncode == 0, " ".join(cmd) + "\n" + (r.stdout + r.stderr)[-6000:]
    return r


@pytest.mark.skipif(shutil.which("cmake") is None or not os.path.exists(NVCC), reason="needs cmake and nvcc")
def test_cmake_build_install_and_consumer(tmp_path):
    build, prefix, consumer = tmp_path / "build", tmp_path / "prefix", tmp_path / "consumer"
    gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    _run(["cmake", "-S", ROOT, "-B", str(build), f"-DCMAKE_CUDA_COMPILER={NVCC}"] + gen, timeout=300)
    _run(["cmake", "--build", str(build), "-j", str(os.cpu_count() or 4)], timeout=1500)
    r = _run([str(build / "bccl_run"), "-np", "2", "--timeout", "120", "--", str(build / "bccl_check"), "check"],
             timeout=180)
    res = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")][-1]
    assert res["failed_all_ranks"] == 0 and res["ranks"] == 2
    _run(["cmake", "--install", str(build), "--prefix", str(prefix)], timeout=120)
    assert (prefix / "include" / "bccl" / "communicator.h").exists()
    consumer.mkdir()
    (consumer / "CMakeLists.txt").write_text(CONSUMER_CMAKE)
    (consumer / "main.cc").write_text(CONSUMER_MAIN)
    _run(["cmake", "-S", str(consumer), "-B", str(consumer / "build"), f"-DCMAKE_PREFIX_PATH={prefix}"] + gen,
         timeout=300)
    _run(["cmake", "--build", str(consumer / "build")], timeout=300)
    r = _run([str(consumer / "build" / "consumer")], timeout=60)
    assert "consumer 1 2 3 4" in r.stdout
