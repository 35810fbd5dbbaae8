"""Benchmark records: every benchmark prints one JSON object per measurement and, with
``--out PATH``, appends the same line to a JSON-lines file (conventionally
``bench/results/<benchmark>.jsonl``), so sweeps from several runs and boxes can be collected and
fed to ``utils/tune.py`` or tabulated. Each appended record carries the benchmark name, a UTC
timestamp, the host name and the GPU name.

The reference's tests print ``OCCL_TEST_RESULT {json}`` lines and append them to a report
(OriginCCL tests/test_common.cpp:479-503); this is the same idea for the benchmarks.
"""
from __future__ import annotations

import json
import os
import socket
import time
from typing import Any, Dict, Optional, Union


def _gpu_name() -> Optional[str]:
    try:
        import torch
        return torch.cuda.get_device_name() if torch.cuda.is_available() else None
    except Exception:  # noqa: BLE001 - a missing or broken CUDA runtime just leaves the field out
        return None


class ResultLog:
    """``log(record)`` prints ``record`` (a dict or an already-encoded JSON line) and appends it,
    with the run's metadata, to ``path`` when one was given. Only ``enabled`` instances (rank 0)
    print or write."""

    def __init__(self, bench: str, path: str = "", enabled: bool = True) -> None:
        self.bench = bench
        self.enabled = enabled
        self._f = None
        self._meta: Dict[str, Any] = {}
        if enabled and path:
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
            self._f = open(path, "a")
            self._meta = {"host": socket.gethostname(), "gpu": _gpu_name()}

    def __call__(self, record: Union[str, Dict[str, Any]]) -> None:
        if not self.enabled:
            return
        line = record if isinstance(record, str) else json.dumps(record)
        print(line, flush=True)
        if self._f is not None:
            full = {"bench": self.bench, "utc": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), **self._meta,
                    **json.loads(line)}
            self._f.write(json.dumps(full) + "\n")
            self._f.flush()

    def close(self) -> None:
        if self._f is not None:
            self._f.close()
            self._f = None

    def __enter__(self) -> "ResultLog":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
