"""Multi-GPU training API (include/dlvk/deployment/multi_gpu_trainer.h:
27-266, include/dlvk/deployment/ring_all_reduce.h:15-81).

The reference drives replicas from threads of one process and its ring
moves no data (src/deployment/ring_all_reduce.cpp:9-271).  Here the same
API runs SPMD, one process per GPU (torchrun / torch.distributed): every
rank builds a `MultiGPUTrainer`, reads its shard of the data (DataLoader
with rank / world_size), and each training step is one captured graph in
which the gradient buckets are all-reduced *and* applied by the fused
NVLink all-reduce + optimizer kernel as soon as backward produces them
(`use_nccl=True` selects NCCL all-reduce + a separate optimizer kernel).
Metrics are summed over ranks with one collective per epoch.

`RingAllReduce` keeps the reference's name and `Stats` fields but is the
framework's P2P all-reduce kernel (one-shot reads of every peer's buffer
through NVLink) timed with CUDA events; bandwidth is reported as bus
bandwidth 2(N-1)/N * bytes / time.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ..parallel.comm import CommunicationBackend, GradientSyncStrategy, NcclBackend, NvlinkBackend
from ..training.callbacks import TrainingMetrics
from ..training.step import TrainStep


def _world():
    return (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)


@dataclass
class MultiGPUConfig:
    device_ids: List[int] = field(default_factory=list)
    master_device: int = 0
    synchronous_updates: bool = True
    gradient_accumulation_steps: int = 1
    use_nccl: bool = False
    communication_overlap: float = 0.5
    bucket_mb: float = 25.0


@dataclass
class TrainingStats:
    total_batches: int = 0
    sync_operations: int = 0
    communication_time: float = 0.0
    computation_time: float = 0.0
    communication_efficiency: float = 0.0
    scaling_efficiency: float = 0.0


class MultiGPUTrainer:
    Config = MultiGPUConfig

    def __init__(self, config: Optional[MultiGPUConfig] = None):
        self.config = config or MultiGPUConfig()
        if not self.config.synchronous_updates:
            raise NotImplementedError("asynchronous updates are not supported; updates are synchronous")
        self.model = None
        self.optimizer = None
        self.loss_fn = None
        self.dp = None
        self._steps = {}
        self.stats = TrainingStats()
        self.world, self.rank = _world()

    def initialize(self, base_model, optimizer=None, loss_fn=None) -> bool:
        """Adopt `base_model` (already on this rank's GPU), wrap it for data
        parallelism; every replica starts from rank 0's parameters."""
        from .. import losses as Lo
        from .. import optim as O

        self.model = base_model.build()
        self.optimizer = optimizer or O.Adam(1e-3)
        self.loss_fn = loss_fn or Lo.CrossEntropyLoss()
        if self.world > 1:
            from ..parallel.data_parallel import DataParallel

            self.dp = DataParallel(self.model, self.optimizer, "nccl" if self.config.use_nccl else "fused",
                                   self.config.bucket_mb)
        return True

    def _step(self, x, y) -> TrainStep:
        key = (tuple(x.shape), x.dtype, tuple(y.shape), y.dtype)
        st = self._steps.get(key)
        if st is None:
            st = TrainStep(self.model, self.loss_fn, self.optimizer, dp=self.dp, metrics=True)
            self._steps[key] = st
        return st

    def _accumulated(self, loader):
        """gradient_accumulation_steps k: k consecutive batches are stepped as
        one k-times larger batch (identical mean-loss gradient)."""
        k = max(1, int(self.config.gradient_accumulation_steps))
        if k == 1:
            yield from loader
            return
        xs, ys = [], []
        for x, y in loader:
            xs.append(x)
            ys.append(y)
            if len(xs) == k:
                yield torch.cat(xs), torch.cat(ys)
                xs, ys = [], []
        if xs:
            yield torch.cat(xs), torch.cat(ys)

    def _reduce(self, vals: Sequence[float]) -> List[float]:
        t = torch.tensor(list(vals), dtype=torch.float64, device=self.model.dev.device)
        if self.world > 1:
            dist.all_reduce(t)
        return t.tolist()

    def train(self, train_loader, val_loader=None, epochs: int = 1, callbacks=()) -> TrainingMetrics:
        for cb in callbacks:
            cb.trainer = self
            cb.on_train_begin()
        m = TrainingMetrics()
        for epoch in range(epochs):
            for cb in callbacks:
                cb.on_epoch_begin(epoch)
            self.model.set_training(True)
            t0 = time.perf_counter()
            nb = 0
            for x, y in self._accumulated(train_loader):
                self._step(x, y)(x, y)
                nb += 1
            loss_sum = correct = samples = rows = 0.0
            for st in self._steps.values():
                r = st.rows
                l_, a_, n_ = st.epoch_metrics()
                loss_sum += l_ * n_
                correct += a_ * r
                samples += n_
                rows += r
            if self.model.dev.is_cuda:
                torch.cuda.synchronize(self.model.dev.device)
            dt = time.perf_counter() - t0
            tot = self._reduce([loss_sum, correct, samples, rows])
            m = TrainingMetrics(loss=tot[0] / max(tot[2], 1), accuracy=tot[1] / max(tot[3], 1), epoch=epoch,
                                learning_rate=self.optimizer.get_learning_rate(), epoch_time_ms=dt * 1e3,
                                samples_per_s=tot[2] / dt if dt > 0 else 0.0)
            self.stats.total_batches += nb
            self.stats.sync_operations += nb * (len(self.dp.buckets) if self.dp else 0)
            self.stats.computation_time += dt
            if val_loader is not None:
                vm = self.evaluate(val_loader)
                m.validation_loss, m.validation_accuracy = vm.loss, vm.accuracy
            for cb in callbacks:
                cb.on_epoch_end(epoch, m)
            if hasattr(train_loader, "new_epoch"):
                train_loader.new_epoch()
        for cb in callbacks:
            cb.on_train_end()
        return m

    def evaluate(self, loader) -> TrainingMetrics:
        self.model.set_training(False)
        fused = getattr(self.loss_fn, "fuses_softmax", False) and self.model.has_trailing_softmax()
        loss_sum = correct = n = rows = 0.0
        with torch.no_grad():
            for x, y in loader:
                out = self.model.forward_logits(x) if fused else self.model.forward(x)
                yd = y.to(out.device)
                loss, _ = self.loss_fn.value_and_grad(out, yd, from_logits=fused)
                loss_sum += float(loss) * x.shape[0]
                n += x.shape[0]
                if out.shape[-1] > 1:
                    p = out.reshape(-1, out.shape[-1]).float().argmax(-1)
                    t = yd.reshape(-1, yd.shape[-1]).argmax(-1) if yd.is_floating_point() else yd.reshape(-1).long()
                    correct += float((p == t).sum())
                    rows += p.numel()
        tot = self._reduce([loss_sum, correct, n, rows])
        return TrainingMetrics(loss=tot[0] / max(tot[2], 1), accuracy=tot[1] / max(tot[3], 1))

    def get_consolidated_model(self):
        """The trained model with complete master weights on every rank
        (collective when sharded optimizer updates are in use)."""
        if self.dp is not None:
            self.dp.consolidate()
        self.model.store.sync_value()
        return self.model

    def get_stats(self) -> TrainingStats:
        return self.stats

    def save_checkpoint(self, checkpoint_path: str) -> bool:
        self.get_consolidated_model()
        if self.rank == 0:
            self.model.save_weights(checkpoint_path, optimizer=self.optimizer)
        if self.world > 1:
            dist.barrier()
        return True

    def load_checkpoint(self, checkpoint_path: str) -> bool:
        self.model.load_weights(checkpoint_path, optimizer=self.optimizer)
        return True

    def close(self) -> None:
        for st in self._steps.values():
            st.close()
        self._steps.clear()
        if self.dp is not None:
            self.dp.close()
            self.dp = None


@dataclass
class DeviceInfo:
    device_id: int
    device_name: str
    memory_size: int
    compute_capability: float
    is_available: bool


class MultiGPUDeviceManager:
    @staticmethod
    def detect_gpus() -> List[DeviceInfo]:
        out = []
        if not torch.cuda.is_available():
            return out
        for i in range(torch.cuda.device_count()):
            p = torch.cuda.get_device_properties(i)
            try:
                free, _ = torch.cuda.mem_get_info(i)
                avail = free > 0
            except RuntimeError:
                avail = False
            out.append(DeviceInfo(i, p.name, int(p.total_memory), float(f"{p.major}.{p.minor}"), avail))
        return out

    @staticmethod
    def estimate_memory_requirements(model, batch_size: int) -> int:
        """fp32 master + fp32 grad + Adam m, v + compute-dtype copy, plus
        activations of the widest layer for `batch_size` samples kept for
        backward in every layer."""
        model.build()
        n = model.parameter_count()
        elt = 2 if model.dtype == torch.bfloat16 else 4
        widest = max([getattr(l, "output_size", 0) or getattr(l, "d_model", 0) or 0 for l in model.m_layers] + [1])
        return int(n * (4 + 4 + 8 + elt) + batch_size * widest * elt * max(1, len(model.m_layers)) * 2)

    @staticmethod
    def select_optimal_config(available_gpus: Sequence[DeviceInfo], model_size: int,
                              batch_size: int) -> MultiGPUConfig:
        ids = [g.device_id for g in available_gpus if g.is_available and g.memory_size > model_size]
        cfg = MultiGPUConfig(device_ids=ids or [0])
        # gradient accumulation only when one replica cannot hold its share of the batch
        per = max(1, batch_size // max(1, len(cfg.device_ids)))
        mem = min((g.memory_size for g in available_gpus), default=0)
        if mem and model_size * 4 > mem:
            cfg.gradient_accumulation_steps = 2
        cfg.use_nccl = False  # the fused NVLink all-reduce + optimizer is the default
        return cfg

    @staticmethod
    def check_compatibility(device_ids: Sequence[int]) -> bool:
        if not torch.cuda.is_available():
            return False
        ids = list(device_ids)
        if any(i >= torch.cuda.device_count() for i in ids):
            return False
        caps = {torch.cuda.get_device_capability(i) for i in ids}
        if len(caps) != 1:
            return False
        for a in ids:
            for b in ids:
                if a != b and not torch.cuda.can_device_access_peer(a, b):
                    return False
        return True


# The reference's Vulkan backend maps to the NVLink P2P backend here.
VulkanCommunicationBackend = NvlinkBackend


class RingAllReduce:
    """All-reduce with measured statistics (ring_all_reduce.h:15-81)."""

    @dataclass
    class Stats:
        total_time_ms: float = 0.0
        transfer_time_ms: float = 0.0
        compute_time_ms: float = 0.0
        bytes_transferred: int = 0
        bandwidth_gbps: float = 0.0

    def __init__(self, devices=None, group=None, use_p2p: bool = True, capacity_bytes: int = 256 << 20):
        self.world, self.rank = _world()
        self.backend: CommunicationBackend = (NvlinkBackend(group, capacity_bytes)
                                              if (use_p2p and torch.cuda.is_available()) else NcclBackend(group))
        self.ok = self.backend.initialize(devices)
        self.stats = RingAllReduce.Stats()

    def perform_all_reduce(self, tensors, average: bool = False) -> None:
        if isinstance(tensors, torch.Tensor):
            tensors = [tensors]
        cuda = tensors[0].is_cuda
        if cuda:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
        t0 = time.perf_counter()
        if self.world > 1:
            self.backend.all_reduce(tensors, average)
        if cuda:
            e.record()
            e.synchronize()
            ms = s.elapsed_time(e)
        else:
            ms = (time.perf_counter() - t0) * 1e3
        nb = sum(t.numel() * t.element_size() for t in tensors)
        moved = int(2 * (self.world - 1) / max(self.world, 1) * nb)
        st = self.stats
        st.total_time_ms += ms
        st.transfer_time_ms += ms
        st.bytes_transferred += moved
        st.bandwidth_gbps = st.bytes_transferred / (st.total_time_ms * 1e-3) / 1e9 if st.total_time_ms > 0 else 0.0

    def get_stats(self) -> "RingAllReduce.Stats":
        return self.stats
