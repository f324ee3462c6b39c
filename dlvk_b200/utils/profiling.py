"""Tracing and device-timed statistics.

The reference timed with std::chrono only and its RingAllReduce::Stats
added hard-coded 0.1 ms / 0.05 ms per step (src/deployment/
ring_all_reduce.cpp:150-160,255,261).  Here:

* `nvtx_range(name)` marks a region for Nsight Systems (no-op when NVTX is
  unavailable); with DLVK_NVTX=1 every layer's forward is wrapped in one
  (models/sequential.py).
* `EventTimer` records CUDA events around named regions on the current
  stream and reports device milliseconds (never a profiler number).
* `Stats` keeps the reference's field names (total_time_ms,
  bytes_transferred, bandwidth_gbps) filled with measured values.
"""
from __future__ import annotations

import contextlib
import os
import time
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

NVTX_LAYERS = os.environ.get("DLVK_NVTX", "0") == "1"


@contextlib.contextmanager
def nvtx_range(name: str):
    pushed = False
    if torch.cuda.is_available():
        try:
            torch.cuda.nvtx.range_push(name)
            pushed = True
        except RuntimeError:
            pushed = False
    try:
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()


@dataclass
class Stats:
    total_time_ms: float = 0.0
    bytes_transferred: int = 0
    operations: int = 0

    @property
    def bandwidth_gbps(self) -> float:
        return self.bytes_transferred / (self.total_time_ms * 1e-3) / 1e9 if self.total_time_ms > 0 else 0.0

    def add(self, ms: float, nbytes: int = 0) -> None:
        self.total_time_ms += ms
        self.bytes_transferred += int(nbytes)
        self.operations += 1

    def as_dict(self) -> dict:
        return {"total_time_ms": self.total_time_ms, "bytes_transferred": self.bytes_transferred,
                "operations": self.operations, "bandwidth_gbps": self.bandwidth_gbps}


class EventTimer:
    """Device-timed named regions:

        t = EventTimer()
        with t("forward"):
            ...
        t.summary()   # {"forward": {"count": n, "total_ms": ..., "mean_ms": ...}}
    """

    def __init__(self, enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self._pending: List[tuple] = []
        self._totals: Dict[str, List[float]] = defaultdict(list)

    @contextlib.contextmanager
    def __call__(self, name: str, nbytes: int = 0):
        if not self.enabled:
            t0 = time.perf_counter()
            yield
            self._totals[name].append((time.perf_counter() - t0) * 1e3)
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        with nvtx_range(name):
            yield
        e.record()
        self._pending.append((name, s, e))

    def _drain(self) -> None:
        for name, s, e in self._pending:
            e.synchronize()
            self._totals[name].append(s.elapsed_time(e))
        self._pending.clear()

    def summary(self) -> Dict[str, dict]:
        self._drain()
        return {k: {"count": len(v), "total_ms": sum(v), "mean_ms": sum(v) / len(v), "max_ms": max(v)}
                for k, v in self._totals.items() if v}

    def reset(self) -> None:
        self._drain()
        self._totals.clear()
