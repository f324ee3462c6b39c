"""Failure detection on the host.

The reference reported errors as bool returns and waited on fences with
UINT64_MAX (src/tensor/tensor_ops.cpp:1686-1709, src/deployment/
ring_all_reduce.cpp:264-271).  Here every device-side wait in this
project's kernels is bounded and, on expiry, records a status code in a
device error word instead of hanging; the host turns that code into an
exception:

* `check_device()` reads (and optionally clears) the error word and raises
  `CommTimeoutError` (a peer never signalled within its budget),
  `PipelineTimeoutError` (an on-chip barrier of a tensor-core kernel never
  completed) or `DeviceError`.
* `wait_event(ev, timeout_s)` polls cudaEventQuery against a deadline
  instead of blocking in cudaEventSynchronize, so a host thread gives up
  on a stuck stream.
* `StepWatchdog` wraps a training step: it records an event after the
  step and raises `StepTimeoutError` if it has not completed in time.
"""
from __future__ import annotations

import time
from typing import Optional

import torch

from .. import _ext

ERR_PEER_TIMEOUT = 1
ERR_BOUNDS = 2
ERR_MBAR_TIMEOUT = 3


class DeviceError(RuntimeError):
    code = 0


class CommTimeoutError(DeviceError):
    """A peer GPU did not signal within the kernel's wait budget."""


class PipelineTimeoutError(DeviceError):
    """A tensor-core kernel's producer/consumer barrier never completed."""


class StepTimeoutError(RuntimeError):
    """A step's work did not finish on the device before the deadline."""


def error_for(code: int) -> Optional[DeviceError]:
    if code == 0:
        return None
    cls = {ERR_PEER_TIMEOUT: CommTimeoutError, ERR_MBAR_TIMEOUT: PipelineTimeoutError}.get(code, DeviceError)
    e = cls(f"device error word = {code}")
    e.code = code
    return e


def check_device(clear: bool = True) -> None:
    """Raise the exception matching the device error word (synchronises)."""
    if not torch.cuda.is_available():
        return
    code = int(_ext.C().read_device_error(clear))
    e = error_for(code)
    if e is not None:
        raise e


def wait_event(ev: "torch.cuda.Event", timeout_s: float, poll_s: float = 1e-4) -> bool:
    """True once `ev` completed; False if the deadline passed first."""
    deadline = time.monotonic() + timeout_s
    while not ev.query():
        if time.monotonic() > deadline:
            return False
        time.sleep(poll_s)
    return True


class StepWatchdog:
    def __init__(self, timeout_s: float = 60.0):
        self.timeout_s = timeout_s

    def __call__(self, fn, *args, **kwargs):
        out = fn(*args, **kwargs)
        if torch.cuda.is_available():
            ev = torch.cuda.Event()
            ev.record()
            if not wait_event(ev, self.timeout_s):
                raise StepTimeoutError(f"step did not complete within {self.timeout_s} s")
            check_device()
        return out
