"""Datasets (include/dlvk/data/dataset.h:16-73, src/data/dataset.cpp).

A `Dataset` exposes `size / get_item / input_shape / target_shape /
num_classes` like the reference.  Datasets that hold their samples as one
contiguous host array additionally expose `arrays()` -> (inputs, labels),
which lets the DataLoader assemble a batch with one native gather into a
pinned buffer instead of per-sample Python calls.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch


class Dataset:
    def size(self) -> int:
        raise NotImplementedError

    def get_item(self, index: int) -> Tuple[torch.Tensor, torch.Tensor]:
        raise NotImplementedError

    def input_shape(self) -> List[int]:
        raise NotImplementedError

    def target_shape(self) -> List[int]:
        return [self.num_classes()]

    def num_classes(self) -> int:
        return 0

    def arrays(self):
        """(inputs [N, ...], labels [N] int32) as contiguous CPU tensors, or
        None when the dataset is not array-backed."""
        return None

    def __len__(self) -> int:
        return self.size()

    def __getitem__(self, i):
        return self.get_item(i)


class TensorDataset(Dataset):
    """In-memory samples: inputs [N, ...] (float32 or uint8) and integer
    class labels [N] (or float targets [N, ...])."""

    def __init__(self, inputs: torch.Tensor, targets: torch.Tensor, num_classes: Optional[int] = None,
                 u8_scale: float = 1.0 / 255.0):
        if inputs.shape[0] != targets.shape[0]:
            raise ValueError("inputs and targets differ in length")
        self.inputs = inputs.contiguous()
        self.targets = targets.contiguous()
        self.u8_scale = u8_scale
        if num_classes is None and not targets.is_floating_point():
            num_classes = int(targets.max()) + 1 if targets.numel() else 0
        self._classes = int(num_classes or 0)

    def size(self) -> int:
        return int(self.inputs.shape[0])

    def get_item(self, index: int):
        x = self.inputs[index]
        if x.dtype == torch.uint8:
            x = x.float() * self.u8_scale
        return x, self.targets[index]

    def input_shape(self):
        return list(self.inputs.shape[1:])

    def target_shape(self):
        return list(self.targets.shape[1:]) if self.targets.is_floating_point() else [self._classes]

    def num_classes(self) -> int:
        return self._classes

    def arrays(self):
        if self.targets.is_floating_point():
            return None
        return self.inputs, self.targets.to(torch.int32).contiguous()


class TransformDataset(Dataset):
    """Applies per-sample transforms on get_item (dataset.cpp:6-42).  The
    DataLoader applies `batch_transform` objects to whole device batches."""

    def __init__(self, dataset: Dataset, input_transform: Optional[Callable] = None,
                 target_transform: Optional[Callable] = None):
        self.base = dataset
        self.input_transform = input_transform
        self.target_transform = target_transform

    def size(self) -> int:
        return self.base.size()

    def get_item(self, index: int):
        x, y = self.base.get_item(index)
        if self.input_transform is not None:
            x = self.input_transform(x)
        if self.target_transform is not None:
            y = self.target_transform(y)
        return x, y

    def input_shape(self):
        if self.input_transform is None:
            return self.base.input_shape()
        return list(self.get_item(0)[0].shape)

    def target_shape(self):
        return self.base.target_shape()

    def num_classes(self) -> int:
        return self.base.num_classes()

    def arrays(self):
        # per-sample transforms run in Python; batch transforms stay on the loader
        return None if (self.input_transform or self.target_transform) else self.base.arrays()


class SyntheticDataset(TensorDataset):
    """Deterministic random samples: U[0,1) inputs, uniform labels."""

    def __init__(self, n: int, input_shape: Sequence[int], num_classes: int, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        x = torch.rand((n, *input_shape), generator=g)
        y = torch.randint(0, num_classes, (n,), generator=g, dtype=torch.int32)
        super().__init__(x, y, num_classes)
