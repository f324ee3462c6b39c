"""DataLoader (include/dlvk/data/dataloader.h:16-89, src/data/dataloader.cpp).

Keeps the reference API (`num_batches`, `get_batch`, iteration,
`new_epoch`, `batch_size`, `dataset_size`, shuffle, drop_last, one-hot
targets) with a different execution model:

* a batch of an array-backed dataset is assembled by the native gather
  (`_C.data`, C++ thread pool, GIL released) straight into a page-locked
  host slot, converting uint8 pixels to fp32 on the way;
* a background thread fills a ring of `prefetch` pinned slots while the
  GPU trains; the host->device copy of the next batch is issued on a
  separate copy stream as soon as the current one is handed out, and the
  consumer stream waits on its event -- so the copy overlaps compute;
* the shuffle is a deterministic permutation of (seed, epoch) computed
  natively; with `world_size > 1` rank r takes every world_size-th
  sample of it, so data-parallel ranks read disjoint shards without
  communicating;
* `batch_transform` (e.g. `transforms.Compose`) runs on the device batch.

The reference supported only MnistDataset (dynamic_cast,
dataloader.cpp:52-58); any `Dataset` works here (array-backed ones take
the native path, others are stacked from `get_item`).
"""
from __future__ import annotations

import queue
import threading
from typing import Callable, Optional

import torch

from .. import _ext


def _as_device(device):
    if device is None:
        return None
    dev = getattr(device, "device", device)
    return torch.device(dev)


class DataLoader:
    def __init__(self, dataset, device=None, batch_size: int = 32, shuffle: bool = True, drop_last: bool = False,
                 seed: int = 0, one_hot: bool = True, prefetch: int = 2, threads: int = 4,
                 batch_transform: Optional[Callable] = None, rank: int = 0, world_size: int = 1,
                 pin_memory: Optional[bool] = None):
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        self.dataset = dataset
        self.device = _as_device(device)
        self._batch_size = int(batch_size)
        self.shuffle = bool(shuffle)
        self.drop_last = bool(drop_last)
        self.seed = int(seed)
        self.one_hot = bool(one_hot)
        self.prefetch = max(1, int(prefetch))
        self.threads = max(1, int(threads))
        self.batch_transform = batch_transform
        self.rank, self.world_size = int(rank), max(1, int(world_size))
        cuda_ok = torch.cuda.is_available()
        self.pin = cuda_ok if pin_memory is None else (bool(pin_memory) and cuda_ok)
        self.epoch = 0
        self.h2d_bytes = 0
        self._arrays = dataset.arrays() if hasattr(dataset, "arrays") else None
        self._classes = max(1, int(dataset.num_classes() or 1))
        self._indices = self._make_indices()
        self._copy_stream = None

    # ------------------------------------------------------------ reference API
    def batch_size(self) -> int:
        return self._batch_size

    def dataset_size(self) -> int:
        return self.dataset.size()

    def num_samples(self) -> int:
        return int(self._indices.numel())

    def num_batches(self) -> int:
        n = self.num_samples()
        return n // self._batch_size if self.drop_last else (n + self._batch_size - 1) // self._batch_size

    __len__ = num_batches

    def new_epoch(self) -> None:
        self.epoch += 1
        self._indices = self._make_indices()

    def get_batch(self, batch_idx: int):
        """Synchronous batch `batch_idx` of the current epoch (device tensors
        when a device was given)."""
        if not 0 <= batch_idx < self.num_batches():
            raise IndexError("batch index out of range")
        hx, hy = self._assemble(batch_idx, None)
        return self._finish(*self._to_device(hx, hy))

    def __iter__(self):
        return _PrefetchIter(self)

    # ------------------------------------------------------------ internals
    def _make_indices(self) -> torch.Tensor:
        n = self.dataset.size()
        if self.shuffle:
            p = _ext.C().data.permutation(n, self.seed, self.epoch)
        else:
            p = torch.arange(n, dtype=torch.int64)
        if self.world_size > 1:
            p = p[self.rank::self.world_size].contiguous()
        return p

    def _batch_index(self, b: int) -> torch.Tensor:
        s = b * self._batch_size
        return self._indices[s:s + self._batch_size].contiguous()

    def _alloc_host(self, n: int):
        if self._arrays is not None:
            xs = tuple(self._arrays[0].shape[1:])
        else:
            xs = tuple(self.dataset.get_item(0)[0].shape)
        x = torch.empty((n, *xs), dtype=torch.float32, pin_memory=self.pin)
        if self.one_hot:
            y = torch.empty((n, self._classes), dtype=torch.float32, pin_memory=self.pin)
        else:
            y = torch.empty((n,), dtype=torch.int32, pin_memory=self.pin)
        return x, y

    def _assemble(self, b: int, slot):
        idx = self._batch_index(b)
        n = int(idx.numel())
        if slot is None or slot[0].shape[0] != n:
            slot = self._alloc_host(n)
        hx, hy = slot
        D = _ext.C().data
        if self._arrays is not None:
            xs, labels = self._arrays
            if xs.dtype == torch.uint8:
                scale = float(getattr(self.dataset, "u8_scale", 1.0 / 255.0))
                D.gather_u8_to_f32(xs, idx, hx, scale, 0.0, self.threads)
            elif xs.dtype == torch.float32:
                D.gather_rows(xs, idx, hx, self.threads)
            else:
                hx.copy_(xs[idx].float())
            if self.one_hot:
                ok = D.gather_labels(labels, idx, self._classes, None, hy)
            else:
                ok = D.gather_labels(labels, idx, self._classes, hy, None)
            if not ok:
                raise ValueError("dataset label outside [0, num_classes)")
        else:
            for i, j in enumerate(idx.tolist()):
                x, y = self.dataset.get_item(j)
                hx[i].copy_(torch.as_tensor(x, dtype=torch.float32).reshape(hx[i].shape))
                if self.one_hot:
                    yt = torch.as_tensor(y)
                    if yt.numel() == self._classes and yt.is_floating_point():
                        hy[i].copy_(yt.reshape(-1))
                    else:
                        hy[i].zero_()
                        hy[i, int(yt)] = 1.0
                else:
                    hy[i] = int(torch.as_tensor(y).reshape(-1)[0])
        return hx, hy

    def _to_device(self, hx, hy, stream=None):
        if self.device is None or self.device.type != "cuda":
            return hx.clone(), hy.clone()
        self.h2d_bytes += hx.nbytes + hy.nbytes
        if stream is None:
            return hx.to(self.device, non_blocking=self.pin), hy.to(self.device, non_blocking=self.pin)
        with torch.cuda.stream(stream):
            dx = torch.empty(hx.shape, dtype=hx.dtype, device=self.device)
            dy = torch.empty(hy.shape, dtype=hy.dtype, device=self.device)
            dx.copy_(hx, non_blocking=True)
            dy.copy_(hy, non_blocking=True)
        return dx, dy

    def _finish(self, x, y):
        if self.batch_transform is not None:
            x = self.batch_transform(x)
        return x, y


class _PrefetchIter:
    """Background host assembly into a ring of pinned slots + one H2D copy
    in flight on a copy stream."""

    def __init__(self, loader: DataLoader):
        self.L = loader
        self.n = loader.num_batches()
        self.next_out = 0
        self.cuda = loader.device is not None and loader.device.type == "cuda"
        self.q: "queue.Queue" = queue.Queue(maxsize=loader.prefetch)
        self.free: "queue.Queue" = queue.Queue()
        for _ in range(loader.prefetch + 1):
            self.free.put(None)  # slots are allocated lazily by the producer
        self.stop = threading.Event()
        self.err = None
        self.inflight = None
        if self.cuda:
            if loader._copy_stream is None:
                loader._copy_stream = torch.cuda.Stream(device=loader.device)
            self.cs = loader._copy_stream
        self.th = threading.Thread(target=self._produce, daemon=True)
        self.th.start()

    def _produce(self):
        try:
            for b in range(self.n):
                if self.stop.is_set():
                    return
                slot = self.free.get()
                if slot is not None and slot[2] is not None:
                    slot[2].synchronize()  # the previous H2D out of this slot finished
                hx, hy = self.L._assemble(b, None if slot is None else (slot[0], slot[1]))
                self.q.put((b, hx, hy))
        except BaseException as e:  # surfaced to the consumer
            self.err = e
            self.q.put(None)

    def _launch(self):
        item = self.q.get()
        if item is None:
            raise self.err
        b, hx, hy = item
        if self.cuda:
            dx, dy = self.L._to_device(hx, hy, self.cs)
            ev = torch.cuda.Event()
            ev.record(self.cs)
            self.free.put((hx, hy, ev))
            return dx, dy, ev
        dx, dy = self.L._to_device(hx, hy)
        self.free.put((hx, hy, None))
        return dx, dy, None

    def __iter__(self):
        return self

    def __next__(self):
        if self.next_out >= self.n:
            self.close()
            raise StopIteration
        cur = self.inflight if self.inflight is not None else self._launch()
        self.inflight = None
        self.next_out += 1
        if self.next_out < self.n:
            self.inflight = self._launch()  # next batch's copy overlaps this batch's compute
        dx, dy, ev = cur
        if ev is not None:
            s = torch.cuda.current_stream(self.L.device)
            s.wait_event(ev)
            dx.record_stream(s)
            dy.record_stream(s)
        return self.L._finish(dx, dy)

    def close(self):
        self.stop.set()
        while self.th.is_alive():
            try:
                self.q.get_nowait()
            except queue.Empty:
                pass
            self.th.join(timeout=0.01)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
