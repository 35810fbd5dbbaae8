"""Samples GPU clocks and throttle reasons with nvidia-smi while a timed region runs.

Usage::

    with ClockSampler(gpu_indices=[0, 1]) as cs:
        ...timed work...
    summary = cs.summary()   # {"sm_mhz": median under load, "sm_max_mhz": ..., "reasons": [...]}

Reading clocks is all it does; it never changes a GPU setting.
"""
from __future__ import annotations

import shutil
import statistics
import subprocess
import threading
import time
from typing import Dict, List, Optional

_FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu",
           "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
           "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, gpu_indices: Optional[List[int]] = None, interval_ms: int = 100) -> None:
        self.gpus = gpu_indices
        self.interval_ms = interval_ms
        self.samples: List[Dict] = []
        self._proc: Optional[subprocess.Popen] = None
        self._thread: Optional[threading.Thread] = None

    def __enter__(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        cmd = [exe, f"--query-gpu={','.join(_FIELDS)}", "--format=csv,noheader,nounits", f"-lms={self.interval_ms}"]
        try:
            self._proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self
        self._thread = threading.Thread(target=self._reader, daemon=True)
        self._thread.start()
        time.sleep(0.05)
        return self

    def _reader(self) -> None:
        assert self._proc is not None and self._proc.stdout is not None
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(_FIELDS):
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

    def __exit__(self, *exc) -> None:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> Dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in self.samples if s["util"] >= 50] or self.samples
        reasons = sorted({r for s in loaded for r in _REASONS if s[r]})
        return {"sm_mhz": statistics.median(s["sm"] for s in loaded),
                "sm_max_mhz": max(s["sm_max"] for s in self.samples),
                "power_w_max": max(s["power"] for s in self.samples),
                "reasons": reasons, "samples": len(self.samples), "samples_under_load": len(loaded)}
