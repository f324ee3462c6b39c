"""Device timing helpers for the kernel micro-benchmarks (CUDA events on the
launching stream, warm-up, L2 flush between timed iterations)."""
from __future__ import annotations

import json
import torch

_FLUSH = None


def flush_l2(nbytes: int = 256 << 20) -> None:
    """Evict L2 (126 MB on B200) by reading a larger buffer, so the next
    launch starts cold.  A read leaves clean lines behind; a write would leave
    dirty ones whose write-back the timed kernel would then pay for."""
    global _FLUSH
    if _FLUSH is None or _FLUSH.numel() * 4 < nbytes:
        _FLUSH = torch.zeros(nbytes // 4, dtype=torch.float32, device="cuda")
    _FLUSH.amax()


def time_fn(fn, iters: int = 20, warmup: int = 3, flush: bool = True) -> float:
    """Median device time of `fn()` in milliseconds.

    Every timed iteration is enqueued before any is waited on, behind a
    ~2 ms spin kernel, so the host runs ahead of the GPU and the events
    bracket device work only (no host launch latency between them).  With
    `flush`, a 256 MB write before each iteration starts it with a cold L2.
    """
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush:
        flush_l2()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    torch.cuda._sleep(4_000_000)
    for s, e in ev:
        if flush:
            flush_l2()
        s.record()
        fn()
        e.record()
    torch.cuda.synchronize()
    times = sorted(s.elapsed_time(e) for s, e in ev)
    return times[len(times) // 2]


def measured_peaks() -> dict:
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}
