"""Samples GPU clocks and throttle reasons while a timed region runs.

Usage::

    with ClockSampler(gpu_indices=[0, 1]) as cs:
        ...timed work...
    summary = cs.summary()   # {"sm_mhz": median under load, "sm_max_mhz": ..., "reasons": [...]}

NVML (``pynvml``) is polled from a thread every ``interval_ms`` (default 20 ms), with one sample
taken on entry and one on exit; without NVML it falls back to ``nvidia-smi -lms``. Reading clocks
is all it does; it never changes a GPU setting.

NVML queries are not free for the GPU being measured: polling several quantities of every GPU
every 2 ms slowed a two-GPU AllReduce loop about fourfold. So the polling thread reads only the
SM clock and the clock-event reasons; the maximum clock and the power draw are read on entry
and on exit, outside the timed work.
"""
from __future__ import annotations

import shutil
import statistics
import subprocess
import threading
import time
from typing import Dict, List, Optional

_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
# NVML clock-event (throttle) reason bits.
_REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
_SMI_FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu",
               "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
               "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


class ClockSampler:
    def __init__(self, gpu_indices: Optional[List[int]] = None, interval_ms: float = 20.0) -> None:
        self.gpus = gpu_indices
        self.interval_ms = interval_ms
        self.samples: List[Dict] = []
        self.source = "none"
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._proc: Optional[subprocess.Popen] = None
        self._nvml = None
        self._handles: List = []

    # ------------------------------------------------------------------ NVML
    def _nvml_start(self) -> bool:
        try:
            import pynvml
            pynvml.nvmlInit()
        except Exception:
            return False
        self._nvml = pynvml
        idx = self.gpus if self.gpus is not None else list(range(pynvml.nvmlDeviceGetCount()))
        try:
            self._handles = [(i, pynvml.nvmlDeviceGetHandleByIndex(i)) for i in idx]
        except Exception:
            return False
        self.source = "nvml"
        self._nvml_sample(full=True)
        self._thread = threading.Thread(target=self._nvml_loop, daemon=True)
        self._thread.start()
        return True

    def _nvml_sample(self, full: bool = False) -> None:
        nv = self._nvml
        for i, h in self._handles:
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                bits = int(get_reasons(h))
                rec = {"index": i, "sm": sm, **{r: bool(bits & _REASON_BITS[r]) for r in _REASONS}}
                if full:
                    rec["sm_max"] = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
                    rec["power"] = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            except Exception:
                continue
            self.samples.append(rec)

    def _nvml_loop(self) -> None:
        while not self._stop.wait(self.interval_ms / 1000.0):
            self._nvml_sample()

    # ------------------------------------------------------------------ nvidia-smi fallback
    def _smi_start(self) -> None:
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return
        cmd = [exe, f"--query-gpu={','.join(_SMI_FIELDS)}", "--format=csv,noheader,nounits",
               f"-lms={max(int(self.interval_ms), 20)}"]
        try:
            self._proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.source = "nvidia-smi"
        self._thread = threading.Thread(target=self._smi_reader, daemon=True)
        self._thread.start()
        time.sleep(0.05)

    def _smi_reader(self) -> None:
        assert self._proc is not None and self._proc.stdout is not None
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(_SMI_FIELDS):
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if self.gpus is not None and idx not in self.gpus:
                continue

            def num(s: str) -> float:
                try:
                    return float(s)
                except ValueError:
                    return float("nan")
            self.samples.append({"index": idx, "sm": num(parts[1]), "sm_max": num(parts[2]), "power": num(parts[3]),
                                 "util": num(parts[4]),
                                 **{r: parts[5 + i] == "Active" for i, r in enumerate(_REASONS)}})

    # ------------------------------------------------------------------ context manager
    def __enter__(self) -> "ClockSampler":
        if self.gpus == []:
            return self
        if not self._nvml_start():
            self._smi_start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if self._nvml is not None:
            self._nvml_sample(full=True)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self) -> Dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        # nvidia-smi samples carry a utilization; NVML polls do not (a utilization query is one
        # more call per poll) and are all taken while the timed work runs.
        loaded = [s for s in self.samples if s.get("util", 100.0) >= 50] or self.samples
        reasons = sorted({r for s in loaded for r in _REASONS if s[r]})
        maxes = [s["sm_max"] for s in self.samples if "sm_max" in s]
        powers = [s["power"] for s in self.samples if "power" in s]
        return {"sm_mhz": statistics.median(s["sm"] for s in loaded),
                "sm_max_mhz": max(maxes) if maxes else None,
                "power_w_max": max(powers) if powers else None,
                "reasons": reasons, "samples": len(self.samples), "samples_under_load": len(loaded),
                "source": self.source}
