"""A whole training step (forward, fused loss, backward, all-reduce,
optimizer) captured once into a CUDA graph and replayed.

This replaces the reference's per-op submit-and-wait-for-idle execution
(src/tensor/tensor_ops.cpp:1673-1710) and its graph-less fit loop
(src/model/model.cpp:223-318): after capture, one step is one
`cudaGraphLaunch`, so small models are not bound by launch latency.

Public use:

    step = TrainStep(model, CrossEntropyLoss(), Adam(1e-3))
    loss = step(x_pinned, y_pinned)      # H2D of the batch, replay, device loss
    print(loss.item())                   # D2H of the loss
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _ext


class TrainStep:
    def __init__(self, model, loss_fn, optimizer, dp=None, graph: bool = True, warmup_eager: int = 2):
        self.model = model.build()
        self.loss_fn = loss_fn
        self.opt = optimizer
        self.dp = dp
        self.use_graph = bool(graph) and model.dev.is_cuda
        self.warmup_eager = warmup_eager
        self.x = None
        self.y = None
        self.loss = None
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self._captured_launches = 0
        self._eager_runs = 0
        self.replays = 0

    # ---------------------------------------------------------------- body
    def _body(self):
        m = self.model
        m.store.zero_grad()
        m.dev.advance_step()
        if self.dp is not None:
            self.dp.begin_step()
        fused = getattr(self.loss_fn, "fuses_softmax", False) and m.has_trailing_softmax()
        out = m.forward_logits(self.x) if fused else m.forward(self.x)
        loss, dout = self.loss_fn.value_and_grad(out, self.y, from_logits=fused)
        torch.autograd.backward(out, dout)
        m.store.finish_backward()
        if self.dp is not None:
            self.dp.finish_step()
        else:
            self.opt.step(m)
        return loss

    # ---------------------------------------------------------------- staging
    def stage(self, x: torch.Tensor, y: torch.Tensor) -> None:
        """Copy a (pinned) host batch into the step's static device buffers."""
        dev = self.model.dev.device
        if self.x is None:
            self.x = torch.empty(x.shape, dtype=x.dtype, device=dev)
            self.y = torch.empty(y.shape, dtype=y.dtype, device=dev)
        if tuple(x.shape) != tuple(self.x.shape) or tuple(y.shape) != tuple(self.y.shape):
            raise ValueError("TrainStep: batch shape changed; create a new TrainStep for a new shape")
        self.x.copy_(x, non_blocking=True)
        self.y.copy_(y, non_blocking=True)

    def run_staged(self) -> torch.Tensor:
        if not self.use_graph:
            self.loss = self._body()
            return self.loss
        if self.graph is None:
            if self._eager_runs < self.warmup_eager:
                # warm-up on a side stream (allocator / autograd state) before capture
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    self.loss = self._body()
                torch.cuda.current_stream().wait_stream(s)
                self._eager_runs += 1
                return self.loss
            self._capture()
        self.graph.replay()
        self.replays += 1
        return self.loss

    def _capture(self):
        torch.cuda.synchronize()
        C = _ext.C()
        g = torch.cuda.CUDAGraph()
        l0 = C.launch_count()
        with torch.cuda.graph(g):
            self.loss = self._body()
        self._captured_launches = C.launch_count() - l0
        self.graph = g
        torch.cuda.synchronize()

    def graph_launches_per_step(self) -> int:
        """Kernels of this project per replayed step (0 in eager mode, where
        the launch counter sees every launch directly)."""
        return self._captured_launches if self.graph is not None else 0

    def __call__(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        self.stage(x, y)
        return self.run_staged()

    def close(self) -> None:
        """Release the captured graph (before tearing down communicators)."""
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None
