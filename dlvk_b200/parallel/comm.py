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


def make_symmetric_multicast(numel: int, dtype: torch.dtype, device: torch.device, group=None):
    """Allocate `numel` elements through PyTorch's symmetric memory (which
    binds every rank's allocation to one NVLink multicast object when the
    node supports it) and wrap the per-rank and multicast addresses in a
    non-owning SymmetricBuffer.  Returns (buffer, keep-alive objects) or
    (None, reason) when symmetric memory or multicast is unavailable.
    Collective."""
    mc, reason = 0, "no NVLink multicast support on this node"
    try:
        import torch.distributed._symmetric_memory as symm_mem

        t = symm_mem.empty(numel, dtype=dtype, device=device)
        grp = group if group is not None else dist.group.WORLD
        hdl = symm_mem.rendezvous(t, grp)
        mc = int(getattr(hdl, "multicast_ptr", 0) or 0)
        ptrs = [int(x) for x in hdl.buffer_ptrs]
    except Exception as exc:  # noqa: BLE001 - any failure means: no NVLS here
        mc, reason = 0, f"symmetric memory unavailable ({type(exc).__name__}: {str(exc)[:120]})"
    # every rank votes (failures included) before any takes the multicast path
    ok = torch.tensor([1 if mc else 0], dtype=torch.int32, device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
    if not int(ok.item()):
        return None, reason
    t.zero_()
    torch.cuda.synchronize(device)
    buf = _ext.C().comm.SymmetricBuffer(ptrs, dist.get_rank(group), numel * t.element_size(), device.index, mc)
    return buf, (t, hdl)


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
        if optimizer.clip_norm is not None or optimizer._clip_bounds() is not None:
            raise ValueError("gradient clipping (by norm or by value) is not supported with the fused all-reduce "
                             "optimizer")
        self.C = _ext.C()
        self.store, self.opt = store, optimizer
        self.world, self.rank, self.group = world, rank, group
        dev = store.device
        self.dev = dev
        n = store.numel
        self.bf16 = store.value is not store.master
        self.algo = algo or os.environ.get("DLVK_AR_ALGO", "auto")
        if self.algo not in ("auto", "push", "pull", "nvls"):
            raise ValueError(f"unknown all-reduce algorithm {self.algo!r}")
        # NVLS: gradient and parameter buffers bound to NVLink multicast
        # objects (PyTorch symmetric memory); otherwise cudaMalloc + IPC.
        self.nvls = False
        self.nvls_reason = "not requested"
        self._keep = []
        if world > 1 and self.algo in ("auto", "nvls") and os.environ.get("DLVK_AR_NVLS", "1") != "0":
            g, kg = make_symmetric_multicast(n, torch.float32, dev, group)
            v, kv = (make_symmetric_multicast(n, torch.bfloat16 if self.bf16 else torch.float32, dev, group)
                     if g is not None else (None, kg))
            if g is not None and v is not None:
                self.grad_buf, self.value_buf, self._keep = g, v, [kg, kv]
                self.nvls, self.nvls_reason = True, "multicast"
            else:
                self.nvls_reason = kv if g is not None else kg
        if self.algo == "nvls" and not self.nvls:
            raise RuntimeError(f"NVLS all-reduce requested but unavailable: {self.nvls_reason}")
        if not self.nvls:
            self.grad_buf = make_symmetric(n * 4, dev, group)
            self.value_buf = make_symmetric(n * (2 if self.bf16 else 4), dev, group)
        self.flag_buf = make_symmetric(MAX_BUCKETS * 2 * world * 4, dev, group)
        self.counters = torch.zeros(MAX_BUCKETS, dtype=torch.int32, device=dev)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=dev)
        self.one_shot_bytes = one_shot_bytes if one_shot_bytes is not None else int(
            os.environ.get("DLVK_ONE_SHOT_BYTES", str((8 << 20) // max(world, 1))))
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.ctas = ctas or int(os.environ.get("DLVK_AR_CTAS", str(6 * sms)))
        self.push_ctas = int(os.environ.get("DLVK_PUSH_CTAS", str(2 * sms)))
        self.nvls_ctas = int(os.environ.get("DLVK_NVLS_CTAS", str(4 * sms)))
        self.st = optimizer.state(store)
        self._bucket_ids = {}
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
        # Pick the form per bucket size from timings on this node (before
        # the model's tensors move into the symmetric buffers).
        self.calibration = None
        if world > 1 and self.algo == "auto" and os.environ.get("DLVK_AR_CALIBRATE", "1") != "0":
            self.calibration = self._calibrate()
        if self.bf16:
            store.rebind(grad=self.grad_buf.tensor(0, n, 0), value=self.value_buf.tensor(1, n, 0))
        else:
            store.rebind(grad=self.grad_buf.tensor(0, n, 0), master=self.value_buf.tensor(0, n, 0))
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
        """The form the bucket [start, end) runs as: ll, one-shot, push, pull
        or nvls.  With a start-up calibration the form measured fastest at
        the nearest calibrated size is used (ll only while its buffer has
        room)."""
        n = end - start
        if self.world == 1:
            return "one-shot"
        if self.calibration:
            import math

            best = min(self.calibration["best"], key=lambda e: abs(math.log(max(n, 1) / e[0])))[1]
            if best == "ll":
                return "ll" if self._ll_slot(start, end) is not None else "one-shot"
            return best
        if n * 4 <= self.one_shot_bytes:
            if self._ll_slot(start, end) is not None:
                return "ll"
            return "one-shot"
        if self.algo == "push":
            if self._push_slot(start, end) is not None:
                return "push"
            raise RuntimeError("push all-reduce: receive buffer or flag table full")
        if self.nvls and self.algo in ("auto", "nvls"):
            return "nvls"
        return "pull"

    def _calibrate(self) -> dict:
        """Time every available form on bucket sizes from 256 KB to 64 MB
        (gradients; the fresh symmetric buffers and scratch optimizer state,
        so no model state is touched), max over ranks, and keep the fastest
        per size.  Collective: every rank runs the same launches."""
        n_all = self.store.numel
        dev = self.dev
        sizes = [s for s in (1 << 16, 1 << 18, 1 << 20, 1 << 22, 1 << 24) if s <= n_all] or [n_all // 64 * 64]
        top = max(sizes)
        master = torch.zeros(n_all, dtype=torch.float32, device=dev)
        m = torch.zeros(top, dtype=torch.float32, device=dev) if self.st.m is not None else None
        v = torch.zeros(top, dtype=torch.float32, device=dev) if self.st.v is not None else None
        slot = MAX_BUCKETS - 1
        table = []
        for size in sizes:
            forms = ["one-shot", "pull"] + (["nvls"] if self.nvls else [])
            if self.ll is not None and size <= self.ll_cap:
                forms.insert(0, "ll")
            times = {}
            for form in forms:
                run = lambda: self._launch(form, 0, size, slot, master, m, v, None, ll_off=0)  # noqa: E731
                for _ in range(2):
                    self.begin_step()
                    run()
                evs = []
                for _ in range(5):
                    self.begin_step()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    run()
                    b.record()
                    evs.append((a, b))
                torch.cuda.synchronize(dev)
                t = sorted(x.elapsed_time(y) for x, y in evs)[2]
                tt = torch.tensor([t], dtype=torch.float64, device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=self.group)
                times[form] = float(tt.item())
            best = min(times, key=times.get)
            table.append((size, best, {k: round(val * 1e3, 2) for k, val in times.items()}))
        if self.C.read_device_error(True) != 0:
            raise RuntimeError("all-reduce calibration: a peer wait timed out")
        self.grad_buf.tensor(0, n_all, 0).zero_()
        self.counters.zero_()
        torch.cuda.synchronize(dev)
        return {"best": [(sz, b) for sz, b, _ in table],
                "us": {str(sz * 4): t for sz, _, t in table}}

    def begin_step(self) -> None:
        self.C.counter_add(self.epoch, 1)

    def reduce_update(self, start: int, end: int, algo: Optional[str] = None, ctas: Optional[int] = None) -> None:
        """Launch the fused all-reduce + update of [start, end) on the current
        stream.  `algo` = "pull" forces the pull two-shot form for a bucket
        that would run push or nvls, "one-shot" the pull one-shot form for
        one that would run ll, "nvls" the multicast form (when available),
        and `ctas` overrides the grid size (all for comparisons)."""
        key = (start, end)
        if key not in self._bucket_ids:
            if len(self._bucket_ids) >= MAX_BUCKETS:
                raise RuntimeError("too many buckets")
            self._bucket_ids[key] = len(self._bucket_ids)
        b = self._bucket_ids[key]
        chosen = self.algorithm(start, end)
        if algo == "pull" and chosen in ("push", "nvls"):
            chosen = "pull"
        if algo == "one-shot" and chosen == "ll":
            chosen = "one-shot"
        if algo == "nvls" and self.nvls:
            chosen = "nvls"
        st = self.st
        self._launch(chosen, start, end, b, self.store.master, st.m, st.v, ctas,
                     ll_off=self._ll.get(key, 0), push=self._push.get(key))

    def _launch(self, algo, start, end, slot, master, m, v, ctas, ll_off=0, push=None) -> None:
        """One fused all-reduce + update of [start, end) in form `algo`, with
        flag / counter slot `slot` and the given fp32 master and optimizer
        state buffers (full-length, or bucket-length starting at `start`)."""
        st = self.st
        if algo == "ll":
            self.C.comm.fused_allreduce_optimizer_ll(
                self.grad_buf, self.value_buf, self.ll, start, end, ll_off, self.ll_cap, master,
                m, v, st.hyper, self.opt.kind, self.epoch, self.world, self.rank, not self.bf16,
                1 if self.bf16 else 0, ctas or self.ctas, BUDGET_S)
        elif algo == "push":
            row, off = push
            self.C.comm.fused_allreduce_optimizer_push(
                self.grad_buf, self.value_buf, self.flag_buf, self.recv, self.cflags, self.counters, slot, row, start,
                end, off, self.recv_slot, master, m, v, st.hyper, self.opt.kind, self.epoch,
                self.world, self.rank, not self.bf16, 0, 1 if self.bf16 else 0, ctas or self.push_ctas, BUDGET_S)
        elif algo == "nvls":
            self.C.comm.fused_allreduce_optimizer_nvls(
                self.grad_buf, self.value_buf, self.flag_buf, self.counters, slot, start, end, master, m, v,
                st.hyper, self.opt.kind, self.epoch, self.world, self.rank, not self.bf16, 1 if self.bf16 else 0,
                ctas or self.nvls_ctas, BUDGET_S)
        else:
            self.C.comm.fused_allreduce_optimizer(
                self.grad_buf, self.value_buf, self.flag_buf, self.counters, slot, start, end, master,
                m, v, st.hyper, self.opt.kind, self.epoch, self.world, self.rank, algo == "one-shot", not self.bf16,
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
    """Every collective on this framework's P2P kernels over NVLink: the
    caller's tensor is staged in a symmetric (IPC-mapped) buffer, ranks
    announce it with ready flags and read each other's staging buffers
    directly (all-reduce: two-shot, each rank sums its shard and stores it to
    all; broadcast / all-gather: pull copies; reduce-scatter: each rank sums
    its chunk in rank order), bounded flag waits throughout.  Tensors larger
    than the staging buffer, or of other dtypes, go through NCCL."""

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

    def _fits(self, t: torch.Tensor) -> bool:
        return t.is_cuda and t.dtype in (torch.float32, torch.bfloat16) and t.numel() * t.element_size() <= self.capacity

    def _collective(self, t: torch.Tensor, out: torch.Tensor, mode: int, root: int = 0) -> None:
        view = self.buf.tensor(_codes(t.dtype), t.numel(), 0)
        view.copy_(t.reshape(-1))
        self.C.counter_add(self.epoch, 1)
        self.C.comm.p2p_collective(self.buf, self.flags, self.counters, 1, out, t.numel(), mode, root, self.epoch,
                                   self.world, self.rank, _codes(t.dtype), 64, BUDGET_S)

    def broadcast(self, tensor, root: int = 0) -> bool:
        if not self._fits(tensor):
            return self.nccl.broadcast(tensor, root)
        out = torch.empty(tensor.numel(), dtype=tensor.dtype, device=tensor.device)
        self._collective(tensor.contiguous(), out, 0, root)
        if self.rank != root:
            tensor.copy_(out.reshape(tensor.shape))
        return True

    def all_gather(self, tensor):
        if not self._fits(tensor):
            return self.nccl.all_gather(tensor)
        out = torch.empty(self.world * tensor.numel(), dtype=tensor.dtype, device=tensor.device)
        self._collective(tensor.contiguous(), out, 1)
        return [c.reshape(tensor.shape) for c in out.chunk(self.world)]

    def reduce_scatter(self, tensor):
        """This rank's chunk of the sum over ranks (chunks as tensor.chunk(world))."""
        if not self._fits(tensor) or tensor.shape[0] % self.world != 0:
            return self.nccl.reduce_scatter(tensor)
        t = tensor.contiguous()
        chunk = t.numel() // self.world
        out = torch.empty(chunk, dtype=t.dtype, device=t.device)
        self._collective(t, out, 2)
        return out.reshape((t.shape[0] // self.world,) + tuple(t.shape[1:]))
