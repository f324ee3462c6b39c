"""Optimizer update overlapped with the backward pass (one GPU).

The flat parameter store is split into contiguous buckets in reverse layer
order, as for data parallelism.  As soon as backward has written the last
gradient of a bucket, that bucket's optimizer update (optim.cu, one launch)
is enqueued on a side stream behind everything already enqueued on the
compute stream, with a capped grid: the memory-bound update then runs beside
the compute-bound backward kernels, whose CTAs leave room for one update CTA
per SM, instead of after them.  The compute stream joins the side stream at
the end of the step, before the next forward reads the parameters.

Same step protocol as parallel.data_parallel.DataParallel (begin_step, the
per-parameter grad-ready hooks, finish_step), so TrainStep(dp=...) drives
it, also inside a captured CUDA graph.  Global-norm clipping, dynamic loss
scaling and regularisers need every gradient before the first update and
are not supported here.

The reference has no counterpart: its optimizers run after backward on the
host thread (src/optimizers/optimizers.cpp, src/optimizers/adam.cpp).
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch

DEFAULT_BUCKET_MB = float(os.environ.get("DLVK_BUCKET_MB", "64"))
DEFAULT_CTAS = int(os.environ.get("DLVK_OVERLAP_CTAS", "148"))


class _Bucket:
    def __init__(self, start: int, end: int, params):
        self.start, self.end, self.params = start, end, params
        self.pending = len(params)


class OverlappedUpdate:
    def __init__(self, model, optimizer, bucket_mb: float = DEFAULT_BUCKET_MB, ctas: Optional[int] = None):
        if optimizer.clip_norm is not None or optimizer._clip_bounds() is not None:
            raise ValueError("gradient clipping needs every gradient before the first update")
        self.model = model.build()
        self.opt = optimizer
        self.store = model.store
        self.dev = model.dev
        self.ctas = DEFAULT_CTAS if ctas is None else int(ctas)
        self.side = self.dev.comm_stream if self.dev.is_cuda else None
        self.buckets = self._make_buckets(bucket_mb)
        self.active = False  # hooks act only between begin_step and finish_step
        self._bucket_of = {}
        for b in self.buckets:
            for p in b.params:
                self._bucket_of[id(p)] = b
                p.on_grad_ready.append(self._on_grad_ready)

    def _make_buckets(self, bucket_mb: float) -> List[_Bucket]:
        limit = int(bucket_mb * (1 << 20) / 4)
        buckets, cur, start, end = [], [], 0, 0
        for p, s, e in self.store.ranges():
            if cur and (e - start) > limit:
                buckets.append(_Bucket(start, end, cur))
                cur, start = [], s
            cur.append(p)
            end = e
        if cur:
            buckets.append(_Bucket(start, self.store.numel, cur))
        return buckets

    def describe(self) -> dict:
        return {"mode": "overlapped-update", "buckets": len(self.buckets), "ctas": self.ctas,
                "bucket_mb": [round((b.end - b.start) * 4 / 2 ** 20, 2) for b in self.buckets]}

    # -------------------------------------------------------- step protocol
    def begin_step(self) -> None:
        for b in self.buckets:
            b.pending = len(b.params)
        self.opt.advance(self.store)
        self.active = True

    def _on_grad_ready(self, p) -> None:
        b = self._bucket_of.get(id(p))
        if b is None or not self.active:
            return
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _launch(self, b: _Bucket) -> None:
        if not self.dev.is_cuda:
            self.opt.update_range(self.store, b.start, b.end)
            return
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            self.opt.update_range(self.store, b.start, b.end, max_ctas=self.ctas)

    def finish_step(self) -> None:
        for b in self.buckets:  # parameters that received no gradient hook
            if b.pending > 0:
                b.pending = 0
                self._launch(b)
        if self.dev.is_cuda:
            torch.cuda.current_stream().wait_stream(self.side)
        self.active = False

    def close(self) -> None:
        for b in self.buckets:
            for p in b.params:
                if self._on_grad_ready in p.on_grad_ready:
                    p.on_grad_ready.remove(self._on_grad_ready)
