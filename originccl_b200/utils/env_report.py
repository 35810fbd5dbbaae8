"""Environment report: the facts a measurement depends on, as one JSON object.

    python -m originccl_b200.utils.env_report

GPU model, count and clocks, driver, CUDA, NCCL and torch versions, NVSwitch multicast support,
the NVLink topology (`nvidia-smi topo -m`) and the library build. Everything is read, nothing is
set; parts that need a GPU are reported as unavailable on a machine without one.
"""
from __future__ import annotations

import json
import os
import platform
import shutil
import subprocess
import sys
from typing import Dict


def _run(cmd) -> str:
    try:
        return subprocess.run(cmd, capture_output=True, text=True, timeout=30).stdout.strip()
    except (OSError, subprocess.TimeoutExpired):
        return ""


def report() -> Dict:
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    out: Dict = {"host": platform.node(), "python": platform.python_version(), "cpus": os.cpu_count()}
    try:
        import torch
        out["torch"] = torch.__version__
        out["torch_cuda"] = torch.version.cuda
        out["cuda_available"] = torch.cuda.is_available()
        if torch.cuda.is_available():
            out["gpus"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
            p = torch.cuda.get_device_properties(0)
            out["sm_count"] = p.multi_processor_count
            out["capability"] = f"{p.major}.{p.minor}"
            out["memory_gb"] = round(p.total_memory / 1e9, 1)
        try:
            out["nccl"] = ".".join(str(v) for v in torch.cuda.nccl.version())
        except Exception:
            out["nccl"] = None
    except ImportError:
        out["torch"] = None
    try:
        import originccl_b200 as occl
        out["bccl"] = occl.version()
        from originccl_b200.ops import gemm
        out["gemm_kernel"] = gemm.kernel_name()
    except Exception as e:  # library not built
        out["bccl"] = f"unavailable: {e}"
    try:
        import pynvml
        pynvml.nvmlInit()
        out["driver"] = pynvml.nvmlSystemGetDriverVersion()
        h = pynvml.nvmlDeviceGetHandleByIndex(0)
        out["sm_max_mhz"] = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        out["power_limit_w"] = pynvml.nvmlDeviceGetPowerManagementLimit(h) / 1000.0
        pynvml.nvmlShutdown()
    except Exception:
        out["driver"] = None
    try:
        from cuda.bindings import driver as cu  # cuda-python
        cu.cuInit(0)
        err, dev = cu.cuDeviceGet(0)
        if err == cu.CUresult.CUDA_SUCCESS:
            err, mc = cu.cuDeviceGetAttribute(cu.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
            out["multicast_supported"] = bool(mc) if err == cu.CUresult.CUDA_SUCCESS else None
    except Exception:
        out["multicast_supported"] = None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out["nvcc"] = (_run([nvcc, "--version"]).splitlines() or [""])[-1] if os.path.exists(nvcc) else None
    smi = shutil.which("nvidia-smi")
    out["topology"] = _run([smi, "topo", "-m"]) if smi else None
    return out


def main() -> int:
    print(json.dumps(report(), indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
