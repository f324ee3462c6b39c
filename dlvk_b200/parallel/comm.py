"""Communication backends (reference `CommunicationBackend`,
include/dlvk/deployment/multi_gpu_trainer.h:222-266: initialize, all_reduce,
broadcast, all_gather, reduce_scatter, finalize).

* `NcclBackend` -- torch.distributed over NCCL (the comparison baseline; also
  gloo on CPU for tests).
* `NvlinkBackend` -- this framework's own kernels over NVLink peer memory
  (symmetric IPC-mapped buffers, P2P loads/stores, bounded flag waits).
* `FusedAllReduceOptimizer` -- the data-parallel gradient path: one kernel per
  bucket that reduces peers' gradients and applies the optimizer (comm.cu).
"""
from __future__ import annotations

import enum
import os
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _ext
from ..ops import core as K


class GradientSyncStrategy(enum.Enum):
    """Reference enum (multi_gpu_trainer.h:212-217); only AllReduce is
    implemented, as in the reference's intent."""
    AllReduce = 0
    ParameterServer = 1
    HierarchicalReduce = 2
    AsyncUpdate = 3


def _codes(dt: torch.dtype) -> int:
    return {torch.float32: 0, torch.bfloat16: 1, torch.int32: 3, torch.int64: 6}[dt]


MAX_BUCKETS = 4096
BUDGET_S = float(os.environ.get("DLVK_PEER_TIMEOUT_S", "10"))


def _exchange(handle: bytes, group=None) -> List[bytes]:
    world = dist.get_world_size(group)
    out = [None] * world
    dist.all_gather_object(out, handle, group=group)
    return out


def make_symmetric(nbytes: int, device: torch.device, group=None):
    """Allocate and map a SymmetricBuffer on every rank (collective)."""
    C = _ext.C()
    buf = C.comm.SymmetricBuffer(int(nbytes), device.index)
    handles = _exchange(buf.handle(), group)
    buf.open(handles, dist.get_rank(group))
    return buf


class FusedAllReduceOptimizer:
    """Per-bucket fused gradient all-reduce + optimizer update.

    The model's flat gradient buffer and compute-dtype parameter buffer are
    moved into symmetric peer-mapped memory.  Buckets smaller than
    `one_shot_bytes` are reduced redundantly on every rank (one round,
    "one-shot"); larger ones two-shot: each rank reduces and updates 1/world
    of the bucket and writes the new parameters to all ranks, so optimizer
    state is touched only by the shard owner.

    One-shot buckets run as "ll" while the LL buffer has room: every rank
    stores its gradients, each value paired with the step epoch in one
    8-byte word, straight into the peers' LL buffers, and receivers poll the
    words themselves -- one NVLink crossing, no flags or barriers -- else as
    "one-shot" (pull, with ready/done flags).  Two-shot comes in two forms:

    * "pull" (default): the owner loads the peers' slices over NVLink with
      6 CTAs of 128 threads per SM, enough loads in flight to cover NVLink
      latency; no extra memory.
    * "push": every rank first stores the gradient slices it does not own
      into the owners' receive buffers, so NVLink carries only stores and the
      reduction reads local memory.  Needs a receive buffer of `recv_factor`
      x (gradient bytes / world) per peer slot.  Measured slower than pull on
      two B200s at every size from 4 MB to 1 GB (its push, fence and reduce
      phases serialise per CTA), so it is opt-in.

    `algo` ("auto", "push", "pull"; env DLVK_AR_ALGO) picks the two-shot
    form; "auto" is pull.  The one-shot threshold defaults to 8 MB / world
    of gradients (LL traffic grows with (world - 1) x 8 bytes per gradient):
    on 8 B200s LL took 19 us for 256 KB where pull two-shot took 35 us for
    1 MB, and on 2 B200s LL took 11 us for 1 MB against 29 us for pull at
    4 MB.
    """

    def __init__(self, store, optimizer, world: int, rank: int, group=None,
                 one_shot_bytes: Optional[int] = None, ctas: Optional[int] = None, algo: Optional[str] = None,
                 recv_factor: Optional[float] = None):
        if optimizer.clip_norm is not None:
            raise ValueError("global-norm clipping is not supported with the fused all-reduce optimizer")
        self.C = _ext.C()
        self.store, self.opt = store, optimizer
        self.world, self.rank, self.group = world, rank, group
        dev = store.device
        self.dev = dev
        n = store.numel
        self.grad_buf = make_symmetric(n * 4, dev, group)
        self.bf16 = store.value is not store.master
        if self.bf16:
            self.value_buf = make_symmetric(n * 2, dev, group)
            store.rebind(grad=self.grad_buf.tensor(0, n, 0), value=self.value_buf.tensor(1, n, 0))
        else:
            self.value_buf = make_symmetric(n * 4, dev, group)
            store.rebind(grad=self.grad_buf.tensor(0, n, 0), master=self.value_buf.tensor(0, n, 0))
        self.flag_buf = make_symmetric(MAX_BUCKETS * 2 * world * 4, dev, group)
        self.counters = torch.zeros(MAX_BUCKETS, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        self.one_shot_bytes = one_shot_bytes if one_shot_bytes is not None else int(
            os.environ.get("DLVK_ONE_SHOT_BYTES", str((8 << 20) // max(world, 1))))
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.ctas = ctas or int(os.environ.get("DLVK_AR_CTAS", str(6 * sms)))
        self.push_ctas = int(os.environ.get("DLVK_PUSH_CTAS", str(2 * sms)))
        self.st = optimizer.state(store)
        self._bucket_ids = {}
        self.algo = algo or os.environ.get("DLVK_AR_ALGO", "auto")
        if self.algo not in ("auto", "push", "pull"):
            raise ValueError(f"unknown all-reduce algorithm {self.algo!r}")
        self._ll = {}  # (start, end) -> LL offset
        self._ll_used = 0
        self.ll = None
        self.ll_cap = 0
        if world > 1 and os.environ.get("DLVK_AR_LL", "1") != "0":
            self.ll_cap = (min(n, self.one_shot_bytes // 4 * 4, int(os.environ.get("DLVK_LL_CAP", str(1 << 22))))
                           + 63) // 64 * 64
            self.ll = make_symmetric(2 * (world - 1) * self.ll_cap * 8, dev, group)
        self._push = {}  # (start, end) -> (flag-table row, receive offset)
        self._recv_used = 0
        self.recv = self.cflags = None
        if world > 1 and self.algo == "push":
            f = recv_factor if recv_factor is not None else float(os.environ.get("DLVK_PUSH_RECV_FACTOR", "2"))
            per = -(-n // world)
            self.recv_slot = (int(f * per) + 64 * self.C.comm.PUSH_MAX_BUCKETS + 63) // 64 * 64
            self.recv = make_symmetric((world - 1) * self.recv_slot * 4, dev, group)
            self.cflags = make_symmetric(self.C.comm.PUSH_MAX_BUCKETS * self.C.comm.PUSH_MAX_CHUNKS * world * 4,
                                         dev, group)
        torch.cuda.synchronize(dev)
        dist.barrier(group)

    def _push_slot(self, start: int, end: int):
        """(flag-table row, receive offset) of a push bucket, or None when the
        receive buffer or the flag table is full (the bucket then runs pull)."""
        key = (start, end)
        if key in self._push:
            return self._push[key]
        if self.recv is None or len(self._push) >= self.C.comm.PUSH_MAX_BUCKETS:
            return None
        shard = ((end - start + self.world - 1) // self.world + 63) // 64 * 64
        if self._recv_used + shard > self.recv_slot:
            return None
        self._push[key] = (len(self._push), self._recv_used)
        self._recv_used += shard
        return self._push[key]

    def _ll_slot(self, start: int, end: int):
        key = (start, end)
        if key in self._ll:
            return self._ll[key]
        if self.ll is None or self._ll_used + (end - start) > self.ll_cap:
            return None
        self._ll[key] = self._ll_used
        self._ll_used += end - start
        return self._ll[key]

    def algorithm(self, start: int, end: int) -> str:
        """The form the bucket [start, end) runs as: ll, one-shot, push or pull."""
        if (end - start) * 4 <= self.one_shot_bytes or self.world == 1:
            if self.world > 1 and self._ll_slot(start, end) is not None:
                return "ll"
            return "one-shot"
        if self.algo == "push":
            if self._push_slot(start, end) is not None:
                return "push"
            raise RuntimeError("push all-reduce: receive buffer or flag table full")
        return "pull"

    def begin_step(self) -> None:
        self.C.counter_add(self.epoch, 1)

    def reduce_update(self, start: int, end: int, algo: Optional[str] = None, ctas: Optional[int] = None) -> None:
        """Launch the fused all-reduce + update of [start, end) on the current
        stream.  `algo` = "pull" forces the pull two-shot form for a bucket
        that would run push, "one-shot" the pull one-shot form for one that
        would run ll, and `ctas` overrides the grid size (both for
        comparisons)."""
        key = (start, end)
        if key not in self._bucket_ids:
            if len(self._bucket_ids) >= MAX_BUCKETS:
                raise RuntimeError("too many buckets")
            self._bucket_ids[key] = len(self._bucket_ids)
        b = self._bucket_ids[key]
        chosen = self.algorithm(start, end)
        if algo == "pull" and chosen == "push":
            chosen = "pull"
        if algo == "one-shot" and chosen == "ll":
            chosen = "one-shot"
        algo = chosen
        st = self.st
        if algo == "ll":
            self.C.comm.fused_allreduce_optimizer_ll(
                self.grad_buf, self.value_buf, self.ll, start, end, self._ll[key], self.ll_cap, self.store.master,
                st.m, st.v, st.hyper, self.opt.kind, self.epoch, self.world, self.rank, not self.bf16,
                1 if self.bf16 else 0, ctas or self.ctas, BUDGET_S)
            return
        if algo == "push":
            row, off = self._push[key]
            self.C.comm.fused_allreduce_optimizer_push(
                self.grad_buf, self.value_buf, self.flag_buf, self.recv, self.cflags, self.counters, b, row, start,
                end, off, self.recv_slot, self.store.master, st.m, st.v, st.hyper, self.opt.kind, self.epoch,
                self.world, self.rank, not self.bf16, 0, 1 if self.bf16 else 0, ctas or self.push_ctas, BUDGET_S)
            return
        one_shot = algo == "one-shot"
        self.C.comm.fused_allreduce_optimizer(
            self.grad_buf, self.value_buf, self.flag_buf, self.counters, b, start, end, self.store.master,
            st.m, st.v, st.hyper, self.opt.kind, self.epoch, self.world, self.rank, one_shot, not self.bf16,
            0, 1 if self.bf16 else 0, ctas or self.ctas, BUDGET_S)

    def close(self) -> None:
        torch.cuda.synchronize(self.dev)


class CommunicationBackend:
    """Interface of the reference (multi_gpu_trainer.h:222-234)."""

    def initialize(self, device_ids=None) -> bool:
        raise NotImplementedError

    def all_reduce(self, tensors, average: bool = False) -> bool:
        raise NotImplementedError

    def broadcast(self, tensor, root: int = 0) -> bool:
        raise NotImplementedError

    def all_gather(self, tensor) -> List[torch.Tensor]:
        raise NotImplementedError

    def reduce_scatter(self, tensor) -> torch.Tensor:
        raise NotImplementedError

    def finalize(self) -> None:
        pass


class NcclBackend(CommunicationBackend):
    """torch.distributed collectives (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        self.group = group

    def initialize(self, device_ids=None) -> bool:
        return dist.is_initialized()

    def all_reduce(self, tensors, average: bool = False) -> bool:
        if isinstance(tensors, torch.Tensor):
            tensors = [tensors]
        w = dist.get_world_size(self.group)
        for t in tensors:
            dist.all_reduce(t, group=self.group)
            if average:
                t.div_(w)
        return True

    def broadcast(self, tensor, root: int = 0) -> bool:
        dist.broadcast(tensor, root, group=self.group)
        return True

    def all_gather(self, tensor) -> List[torch.Tensor]:
        out = [torch.empty_like(tensor) for _ in range(dist.get_world_size(self.group))]
        dist.all_gather(out, tensor, group=self.group)
        return out

    def reduce_scatter(self, tensor) -> torch.Tensor:
        w = dist.get_world_size(self.group)
        chunks = list(tensor.chunk(w))
        out = torch.empty_like(chunks[dist.get_rank(self.group)])
        dist.reduce_scatter(out, chunks, group=self.group)
        return out


class NvlinkBackend(CommunicationBackend):
    """All-reduce through this framework's P2P kernel over a symmetric staging
    buffer (sized on first use); other collectives through NCCL."""

    def __init__(self, group=None, capacity_bytes: int = 256 << 20):
        self.group = group
        self.capacity = capacity_bytes
        self.buf = None
        self.flags = None
        self.nccl = NcclBackend(group)

    def initialize(self, device_ids=None) -> bool:
        if not dist.is_initialized():
            return False
        dev = torch.device("cuda", torch.cuda.current_device())
        w = dist.get_world_size(self.group)
        self.world, self.rank = w, dist.get_rank(self.group)
        self.buf = make_symmetric(self.capacity, dev, self.group)
        self.flags = make_symmetric(2 * w * 4 * 4, dev, self.group)
        self.counters = torch.zeros(4, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        self.C = _ext.C()
        return True

    def all_reduce(self, tensors, average: bool = False) -> bool:
        if isinstance(tensors, torch.Tensor):
            tensors = [tensors]
        for t in tensors:
            nb = t.numel() * t.element_size()
            if nb > self.capacity or t.dtype not in (torch.float32, torch.bfloat16):
                self.nccl.all_reduce([t], average)
                continue
            view = self.buf.tensor(_codes(t.dtype), t.numel(), 0)
            view.copy_(t.reshape(-1))
            self.C.counter_add(self.epoch, 1)
            self.C.comm.p2p_allreduce(self.buf, self.flags, self.counters, 0, 0, t.numel(), self.epoch, self.world,
                                      self.rank, _codes(t.dtype), average, 64, BUDGET_S)
            t.reshape(-1).copy_(view)
        return True

    def broadcast(self, tensor, root: int = 0) -> bool:
        return self.nccl.broadcast(tensor, root)

    def all_gather(self, tensor):
        return self.nccl.all_gather(tensor)

    def reduce_scatter(self, tensor):
        return self.nccl.reduce_scatter(tensor)
