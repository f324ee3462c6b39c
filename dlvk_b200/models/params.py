"""Parameters and their flat storage.

Every trainable tensor of a model lives in three flat, 256-byte aligned
buffers owned by a :class:`ParamStore`:

* ``master`` (fp32) -- the optimizer's copy,
* ``value`` (compute dtype; the same buffer as ``master`` in fp32 mode, a
  bf16 mirror in bf16 mode) -- what the kernels read,
* ``grad`` (fp32) -- where backward kernels write dW/db directly.

Parameters are laid out in *reverse* registration order, so gradients, which
become ready from the last layer to the first, fill the flat gradient buffer
front to back: a data-parallel bucket is a contiguous slice that is complete
as soon as backward has passed its layers.  The optimizer updates the whole
buffer with one kernel launch (or one per bucket, fused with the gradient
all-reduce).
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional

import torch

ALIGN_ELEMS = 64  # 256 bytes of fp32


class Parameter:
    """One trainable tensor (a view into the ParamStore once packed)."""

    def __init__(self, name: str, shape, init: Optional[torch.Tensor] = None, decay: bool = True):
        self.name = name
        self.shape = tuple(int(s) for s in shape)
        self.numel = int(math.prod(self.shape)) if self.shape else 1
        self.master = init.detach().clone().float() if init is not None else torch.zeros(self.shape)
        self.value = self.master
        self.grad = None
        self.decay = decay
        self.offset = -1
        self.fresh = True      # next gradient write overwrites (beta = 0) instead of accumulating
        self.store = None
        self.on_grad_ready: List[Callable[["Parameter"], None]] = []

    # gradient bookkeeping -------------------------------------------------
    def take_accumulate_flag(self) -> bool:
        """True if the next gradient write must accumulate; marks the grad as written."""
        acc = not self.fresh
        self.fresh = False
        return acc

    def grad_ready(self) -> None:
        for cb in self.on_grad_ready:
            cb(self)

    def ensure_grad(self) -> torch.Tensor:
        if self.grad is None:
            self.grad = torch.zeros(self.shape, dtype=torch.float32, device=self.master.device)
        return self.grad

    def __repr__(self) -> str:
        return f"Parameter({self.name}, {self.shape})"


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class ParamStore:
    """Flat storage for a list of parameters (see module docstring)."""

    def __init__(self, params: List[Parameter], device, compute_dtype=torch.float32):
        self.params = list(params)
        self.device = torch.device(device)
        self.compute_dtype = compute_dtype
        order = list(reversed(self.params))
        off = 0
        for p in order:
            p.offset = off
            off += _round_up(p.numel, ALIGN_ELEMS)
        self.numel = max(off, ALIGN_ELEMS)
        self.order = order
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=self.device)
        if compute_dtype == torch.float32:
            self.value = self.master
        else:
            self.value = torch.zeros(self.numel, dtype=compute_dtype, device=self.device)
        for p in order:
            src = p.master.to(self.device, torch.float32).reshape(-1)
            self.master[p.offset:p.offset + p.numel].copy_(src)
            self._bind(p)
        self.sync_value()

    def _bind(self, p: Parameter) -> None:
        sl = slice(p.offset, p.offset + p.numel)
        p.master = self.master[sl].view(p.shape)
        p.value = self.value[sl].view(p.shape)
        p.grad = self.grad[sl].view(p.shape)
        p.store = self

    def rebind(self, grad: torch.Tensor = None, value: torch.Tensor = None, master: torch.Tensor = None) -> None:
        """Move the flat buffers into caller-provided storage (e.g. peer-mapped
        memory for the fused all-reduce), copying current contents."""
        if master is not None:
            master.copy_(self.master)
            if self.value is self.master:
                self.value = master
            self.master = master
        if grad is not None:
            grad.copy_(self.grad)
            self.grad = grad
        if value is not None and self.value is not self.master:
            value.copy_(self.value)
            self.value = value
        for p in self.order:
            self._bind(p)

    def sync_value(self) -> None:
        """Refresh the compute-dtype mirror from the fp32 master."""
        if self.value is not self.master:
            self.value.copy_(self.master)

    def zero_grad(self, set_to_zero: bool = False) -> None:
        for p in self.params:
            p.fresh = True
        if set_to_zero:
            self.grad.zero_()

    def finish_backward(self) -> None:
        """Zero the gradients of parameters that received none this step."""
        for p in self.params:
            if p.fresh:
                p.grad.zero_()
                p.fresh = False

    def ranges(self):
        """(param, start, end) in flat-buffer order."""
        return [(p, p.offset, p.offset + p.numel) for p in self.order]
