"""Data parallelism (reference MultiGPUTrainer, include/dlvk/deployment/
multi_gpu_trainer.h:27-156, whose replicas only slept and whose ring
all-reduce moved no data, src/deployment/multi_gpu_trainer.cpp:167-221,
src/deployment/ring_all_reduce.cpp:141-271).

One process per GPU.  Parameters are replicated; the flat gradient buffer is
split into contiguous buckets in reverse layer order (see params.ParamStore),
and each bucket's reduction starts on the communication stream as soon as
backward has produced its last gradient, overlapping the rest of backward:

* mode "fused": one kernel per bucket reads every peer's gradient slice over
  NVLink (peer pointers exchanged once), reduces in fp32, scales by 1/N and
  applies the optimizer update (comm.cu) -- no separate all-reduce, no
  separate optimizer pass;
* mode "nccl": NCCL all-reduce of the bucket, then this framework's
  optimizer kernel over the bucket -- the comparison baseline.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops import core as K

DEFAULT_BUCKET_MB = float(os.environ.get("DLVK_BUCKET_MB", "64"))
# The parameters whose gradients become ready last (up to one bucket's worth,
# params larger than a bucket excepted) go into smaller buckets, so that
# most of them are reduced while the last layer's backward still runs
# instead of after it (0 disables).
TAIL_BUCKET_MB = float(os.environ.get("DLVK_TAIL_BUCKET_MB", "16"))


class Bucket:
    def __init__(self, idx: int, start: int, end: int, params):
        self.idx, self.start, self.end = idx, start, end
        self.params = params
        self.pending = len(params)
        self.event = None

    @property
    def numel(self) -> int:
        return self.end - self.start


class DataParallel:
    def __init__(self, model, optimizer, mode: str = "fused", bucket_mb: float = DEFAULT_BUCKET_MB,
                 group=None):
        if not dist.is_initialized():
            raise RuntimeError("DataParallel needs torch.distributed initialised (one process per GPU)")
        self.model = model.build()
        self.opt = optimizer
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.store = model.store
        self.dev = model.dev
        self.comm_stream = self.dev.comm_stream if self.dev.is_cuda else None
        self.mode = mode
        self.buckets = self._make_buckets(bucket_mb)
        self._bucket_of = {}
        for b in self.buckets:
            for p in b.params:
                self._bucket_of[id(p)] = b
                p.on_grad_ready.append(self._on_grad_ready)
        self._tl = None  # timeline records while enabled (eager steps only)
        self.fused = None
        if mode == "fused":
            from .comm import FusedAllReduceOptimizer

            self.fused = FusedAllReduceOptimizer(self.store, optimizer, self.world, self.rank, group)
        # make every replica start from rank 0's parameters
        dist.broadcast(self.store.master, 0, group=group)
        self.store.sync_value()
        if self.dev.is_cuda:
            torch.cuda.synchronize(self.dev.device)

    def _make_buckets(self, bucket_mb: float) -> List[Bucket]:
        limit = int(bucket_mb * (1 << 20) / 4)
        tail_limit = int(TAIL_BUCKET_MB * (1 << 20) / 4)
        ranges = self.store.ranges()
        tail, acc = set(), 0
        if 0 < tail_limit < limit:
            for p, s, e in reversed(ranges):  # flat order ends with the first layer: ready last
                if e - s > limit:
                    continue
                if acc + (e - s) > limit:
                    break
                tail.add(id(p))
                acc += e - s
        # Buckets tile the flat store without gaps: each one ends where the
        # next parameter starts, so it also covers the 64-element alignment
        # padding after its last parameter (zero gradients, values that stay
        # zero) and every bucket is a whole number of 64-element blocks.
        buckets, cur, start = [], [], 0
        in_tail = False
        for p, s, e in ranges:
            lim = tail_limit if id(p) in tail else limit
            if cur and ((e - start) > lim or (id(p) in tail) != in_tail):
                buckets.append(Bucket(len(buckets), start, s, cur))
                cur, start = [], s
            in_tail = id(p) in tail
            cur.append(p)
        if cur:
            buckets.append(Bucket(len(buckets), start, self.store.numel, cur))
        return buckets

    def describe(self) -> dict:
        d = {"mode": self.mode, "buckets": len(self.buckets),
             "bucket_mb": [round(b.numel * 4 / 2 ** 20, 2) for b in self.buckets]}
        if self.fused is not None:
            f = self.fused
            d["forms"] = [f.algorithm(b.start, b.end) for b in self.buckets]
            d["nvls"] = f.nvls if f.nvls else f.nvls_reason
            if f.calibration:
                d["calibration_us"] = f.calibration["us"]
        return d

    # ------------------------------------------------------------ step protocol
    # ------------------------------------------------------------ timeline
    def record_timeline(self, on: bool = True) -> None:
        """Record CUDA events per bucket (ready on the compute stream, start
        and end on the comm stream) for the next eager steps; read them with
        timeline().  Events cannot be recorded inside a CUDA-graph capture."""
        self._tl = [] if on else None

    def _ev(self, stream=None):
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    def timeline(self) -> list:
        """Per bucket of the last recorded step: size, form and the ready /
        start / end times (ms from the step's start on this rank)."""
        if not self._tl:
            return []
        torch.cuda.synchronize(self.dev.device)
        t0 = self._tl[0][1]
        out = []
        for kind, ev, b, form in self._tl[1:]:
            out.append({"event": kind, "bucket": b, "form": form, "ms": round(t0.elapsed_time(ev), 4)})
        return out

    def begin_step(self) -> None:
        if self._tl is not None and self.dev.is_cuda:
            self._tl = [("step_start", self._ev(), -1, None)]
        for b in self.buckets:
            b.pending = len(b.params)
        self.opt.advance(self.store)
        if self.fused is not None:
            self.fused.begin_step()

    def _on_grad_ready(self, p) -> None:
        b = self._bucket_of[id(p)]
        b.pending -= 1
        if b.pending == 0:
            self._launch(b)

    def _reduce_bucket(self, b: Bucket) -> None:
        if self.fused is not None:
            self.fused.reduce_update(b.start, b.end)
        else:
            g = self.store.grad[b.start:b.end]
            dist.all_reduce(g, group=self.group)
            self.opt.update_range(self.store, b.start, b.end, extra_scale=1.0 / self.world)

    def _launch(self, b: Bucket) -> None:
        if not self.dev.is_cuda:
            self._reduce_bucket(b)
            return
        cur = torch.cuda.current_stream()
        tl = self._tl is not None and len(self._tl) > 0
        form = self.fused.algorithm(b.start, b.end) if (tl and self.fused is not None) else self.mode
        if tl:
            self._tl.append(("ready", self._ev(cur), b.idx, form))
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            if tl:
                self._tl.append(("start", self._ev(self.comm_stream), b.idx, form))
            self._reduce_bucket(b)
            if tl:
                self._tl.append(("end", self._ev(self.comm_stream), b.idx, form))

    def finish_step(self) -> None:
        # Buckets whose params got no gradient hook call (unused params) are
        # launched here, in bucket order, identically on every rank.
        for b in self.buckets:
            if b.pending > 0:
                b.pending = 0
                self._launch(b)
        if self.dev.is_cuda:
            if self._tl:
                self._tl.append(("backward_end", self._ev(), -1, None))
            torch.cuda.current_stream().wait_stream(self.comm_stream)
            if self._tl:
                self._tl.append(("step_end", self._ev(), -1, None))

    def consolidate(self) -> None:
        """Make every rank's fp32 master and optimizer state complete (two-shot
        buckets update them only on the shard owner).  Call before saving a
        checkpoint; collective."""
        if self.fused is None:
            return
        st = self.opt.state(self.store)
        w = self.world
        for b in self.buckets:
            n = b.numel
            if self.fused.algorithm(b.start, b.end) in ("ll", "one-shot"):
                continue
            shard = ((n + w - 1) // w + 63) // 64 * 64
            for buf in (self.store.master, st.m, st.v):
                if buf is None:
                    continue
                full = torch.zeros(shard * w, dtype=buf.dtype, device=buf.device)
                lo = min(n, shard * self.rank)
                hi = min(n, lo + shard)
                mine = torch.zeros(shard, dtype=buf.dtype, device=buf.device)
                mine[: hi - lo].copy_(buf[b.start + lo:b.start + hi])
                dist.all_gather_into_tensor(full, mine, group=self.group)
                buf[b.start:b.end].copy_(full[:n])
        if self.dev.is_cuda:
            torch.cuda.synchronize(self.dev.device)

    def close(self) -> None:
        if self.fused is not None:
            self.fused.close()
            self.fused = None
