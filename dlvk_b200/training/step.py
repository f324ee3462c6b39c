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

import os

from typing import Optional

import torch

from .. import _ext
from ..ops import core as K


class TrainStep:
    """`scaler` (a GradientScaler) adds device-side dynamic loss scaling,
    `regularizer` (a RegularizationManager) adds fused L1/L2 penalty
    gradients, `metrics=True` accumulates loss x batch and the number of
    correct argmax predictions into device counters (`epoch_metrics()` reads
    and resets them) -- all inside the captured graph."""

    def __init__(self, model, loss_fn, optimizer, dp=None, graph: bool = True, warmup_eager: int = 2,
                 scaler=None, regularizer=None, metrics: bool = False, overlap_update: Optional[bool] = None):
        self.model = model.build()
        self.loss_fn = loss_fn
        self.opt = optimizer
        # One GPU, opt-in (overlap_update=True or DLVK_OVERLAP_UPDATE=1): the
        # optimizer update runs per bucket beside the backward pass
        # (training/overlap.py) when nothing needs all gradients first.  Off by
        # default: on the 12-layer d1024 transformer the update's HBM traffic
        # slowed the backward kernels more than it hid (14.5 vs 13.7 ms/step);
        # a 3 x 4096 MLP gained 4%.
        if overlap_update is None:
            overlap_update = os.environ.get("DLVK_OVERLAP_UPDATE", "0") != "0"
        if (dp is None and overlap_update and model.dev.is_cuda and scaler is None and regularizer is None
                and optimizer.clip_norm is None and optimizer._clip_bounds() is None):
            from .overlap import OverlappedUpdate

            dp = OverlappedUpdate(self.model, optimizer)
            self._own_dp = True
        else:
            self._own_dp = False
        self.dp = dp
        if dp is not None and (scaler is not None or regularizer is not None):
            raise ValueError("with DataParallel use the optimizer's weight_decay; loss scaling and "
                             "regularizers act on local gradients after the bucket all-reduce has started")
        self.scaler = scaler if (scaler is not None and scaler.enabled) else None
        self.regularizer = regularizer
        self.metrics = bool(metrics)
        dev = model.dev.device
        self.loss_sum = torch.zeros(1, dtype=torch.float32, device=dev) if metrics else None
        self.correct = torch.zeros(1, dtype=torch.int64, device=dev) if metrics else None
        self.samples = 0
        self.rows = 0
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
        if self.metrics:
            self._record_metrics(out, loss)
        if self.scaler is not None:
            self.scaler.scale_grad_output(dout)
        torch.autograd.backward(out, dout)
        m.store.finish_backward()
        if self.regularizer is not None:
            self.regularizer.apply_to_store(m.store, self.scaler.scale if self.scaler is not None else None)
        if self.dp is not None:
            self.dp.finish_step()
        else:
            if self.scaler is not None:
                self.scaler.unscale_gradients(self.opt, m.store)
            self.opt.step(m)
            if self.scaler is not None:
                self.scaler.update()
        return loss

    def _record_metrics(self, out, loss):
        rows = out.numel() // out.shape[-1]
        classify = out.shape[-1] > 1
        y = self.y
        if out.is_cuda:
            labels = probs = None
            if classify:
                if y.is_floating_point() and y.numel() == out.numel():
                    probs = y.reshape(rows, -1)
                elif not y.is_floating_point():
                    labels = y.reshape(rows)
            K.N().step_metrics(out.detach().contiguous(), labels, probs, loss.reshape(1), self.loss_sum,
                               self.correct if classify else None, float(self.x.shape[0]))
        else:
            self.loss_sum += loss.detach().float().reshape(1) * self.x.shape[0]
            if classify:
                pred = out.detach().reshape(rows, -1).float().argmax(-1)
                lab = y.reshape(rows, -1).argmax(-1) if y.is_floating_point() else y.reshape(rows).long()
                self.correct += (pred == lab).sum()

    def epoch_metrics(self, reset: bool = True):
        """(mean loss per sample, accuracy per predicted row, samples) since
        the last reset; one D2H read."""
        if not self.metrics:
            raise RuntimeError("TrainStep(metrics=True) is required")
        vals = torch.stack([self.loss_sum.double().reshape(()), self.correct.double().reshape(())]).cpu()
        out = (float(vals[0]) / max(self.samples, 1), float(vals[1]) / max(self.rows, 1), self.samples)
        if reset:
            self.loss_sum.zero_()
            self.correct.zero_()
            self.samples = 0
            self.rows = 0
        return out

    # ---------------------------------------------------------------- staging
    def stage(self, x: torch.Tensor, y: torch.Tensor) -> None:
        """Copy a (pinned) host batch into the step's static device buffers."""
        dev = self.model.dev.device
        if not y.is_floating_point() and y.dtype != torch.int32:
            y = y.to(torch.int32)  # class ids: the fused loss and metrics read int32
        if self.x is None:
            self.x = torch.empty(x.shape, dtype=x.dtype, device=dev)
            self.y = torch.empty(y.shape, dtype=y.dtype, device=dev)
        if tuple(x.shape) != tuple(self.x.shape) or tuple(y.shape) != tuple(self.y.shape):
            raise ValueError("TrainStep: batch shape changed; create a new TrainStep for a new shape")
        self.samples += int(x.shape[0]) if x.dim() else 1
        if y.is_floating_point():
            self.rows += y.numel() // y.shape[-1] if y.dim() > 1 else y.numel()
        else:
            self.rows += y.numel()
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
        if self._own_dp and self.dp is not None:
            self.dp.close()
            self.dp = None
