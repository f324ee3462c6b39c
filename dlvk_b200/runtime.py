"""Device runtime: the CUDA replacement of the reference's `VulkanDevice`
(include/dlvk/core/vulkan_device.h:23-94, src/core/vulkan_device.cpp:15-281)
and of its compute-pipeline manager.

One `CudaDevice` per GPU holds the compute and communication streams, the
device-side RNG step counter used by dropout (so captured graphs draw fresh
masks on each replay), and device queries.  Memory comes from PyTorch's
caching allocator, which replaces the reference's (missing) MemoryPoolManager.
On machines without a GPU the same object drives the CPU reference path.
"""
from __future__ import annotations

import threading
from typing import Dict, Optional

import torch

from . import _ext


class CudaDevice:
    def __init__(self, device: Optional[str | int | torch.device] = None, seed: int = 0):
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        if isinstance(device, int):
            device = torch.device("cuda", device)
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.seed = int(seed)
        self._initialized = False
        self._stream_ids = 0
        self.compute_stream = None
        self.comm_stream = None
        self.step_t = None

    # -- lifecycle (VulkanDevice::initialize / cleanup) ----------------------
    def initialize(self) -> bool:
        if self._initialized:
            return True
        if self.is_cuda:
            _ext.C()  # the native extension is mandatory on a GPU
            torch.cuda.set_device(self.device)
            self.compute_stream = torch.cuda.current_stream(self.device)
            self.comm_stream = torch.cuda.Stream(self.device, priority=-1)
        self.step_t = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._initialized = True
        return True

    def cleanup(self) -> None:
        if self.is_cuda and self._initialized:
            torch.cuda.synchronize(self.device)
        self._initialized = False

    @property
    def is_cuda(self) -> bool:
        return self.device.type == "cuda"

    # -- RNG -----------------------------------------------------------------
    def next_stream_id(self) -> int:
        """A fresh Philox stream id for one dropout site."""
        self._stream_ids += 1
        return self._stream_ids

    def advance_step(self, delta: int = 1) -> None:
        """Advance the device RNG step (stream-ordered, graph-capturable)."""
        self.initialize()
        if self.is_cuda:
            _ext.C().counter_add(self.step_t, int(delta))
        else:
            self.step_t += int(delta)

    # -- queries (VulkanDevice::get_*) ----------------------------------------
    def get_device_name(self) -> str:
        return torch.cuda.get_device_name(self.device) if self.is_cuda else "cpu"

    def get_compute_capability(self):
        return torch.cuda.get_device_capability(self.device) if self.is_cuda else (0, 0)

    def get_sm_count(self) -> int:
        return torch.cuda.get_device_properties(self.device).multi_processor_count if self.is_cuda else 0

    def get_device_type_string(self) -> str:
        if not self.is_cuda:
            return "cpu"
        pr = torch.cuda.get_device_properties(self.device)
        return f"CUDA GPU sm_{pr.major}{pr.minor}, {pr.multi_processor_count} SMs"

    def get_vulkan_version_string(self) -> str:
        """The CUDA runtime version (the reference reported its Vulkan API version)."""
        return f"CUDA {torch.version.cuda}" if self.is_cuda else "cpu"

    def get_max_workgroup_size(self) -> int:
        """Max threads per block (1024 on every GPU this library targets)."""
        return 1024 if self.is_cuda else 0

    def get_total_device_memory(self) -> int:
        return int(torch.cuda.get_device_properties(self.device).total_memory) if self.is_cuda else 0

    def get_max_memory_allocation(self) -> int:
        return self.get_total_device_memory()

    def get_memory_heap_count(self) -> int:
        return 1 if self.is_cuda else 0

    def get_memory_info(self):
        """(free_bytes, total_bytes)."""
        if self.is_cuda:
            return torch.cuda.mem_get_info(self.device)
        return (0, 0)

    def synchronize(self) -> None:
        if self.is_cuda:
            torch.cuda.synchronize(self.device)

    def create_buffer(self, nbytes: int) -> torch.Tensor:
        """Raw device buffer (VulkanDevice::create_buffer)."""
        return torch.empty(int(nbytes), dtype=torch.uint8, device=self.device)

    def __repr__(self) -> str:
        return f"CudaDevice({self.device})"


class ModelContext(CudaDevice):
    """A model's view of its device: its own Philox seed, dropout stream ids
    and device step counter, so the dropout masks of a model depend only on
    that model (seed, order of its dropout sites, its own step count) and not
    on how many other models the process has built or trained on the same
    device.  Streams, queries and everything else are the shared device's."""

    def __init__(self, base: CudaDevice, seed: int = 0):
        self._base = base.base if isinstance(base, ModelContext) else base
        self.device = self._base.device
        self.seed = int(seed)
        self._stream_ids = 0
        self._step_t = None

    @property
    def base(self) -> CudaDevice:
        return self._base

    @property
    def compute_stream(self):
        return self._base.compute_stream

    @property
    def comm_stream(self):
        return self._base.comm_stream

    @property
    def _initialized(self) -> bool:
        return self._base._initialized

    def initialize(self) -> bool:
        ok = self._base.initialize()
        if self._step_t is None:
            self._step_t = torch.zeros(1, dtype=torch.int64, device=self.device)
        return ok

    @property
    def step_t(self):
        if self._step_t is None:
            self.initialize()
        return self._step_t

    def advance_step(self, delta: int = 1) -> None:
        self.initialize()
        if self.is_cuda:
            _ext.C().counter_add(self._step_t, int(delta))
        else:
            self._step_t += int(delta)

    def cleanup(self) -> None:
        self._base.cleanup()

    def __repr__(self) -> str:
        return f"ModelContext({self.device}, seed={self.seed})"


_lock = threading.Lock()
_devices: Dict[str, CudaDevice] = {}


def get_device(device=None) -> CudaDevice:
    """Process-wide CudaDevice for `device` (default: current CUDA device or CPU)."""
    d = CudaDevice(device)
    key = str(d.device)
    with _lock:
        if key not in _devices:
            d.initialize()
            _devices[key] = d
        return _devices[key]
