"""MNIST (include/dlvk/data/mnist.h:13-49, src/data/mnist.cpp).

Reads `train-images-idx3-ubyte` / `train-labels-idx1-ubyte` (or the
`t10k-` pair) with the native IDX reader; pixels stay uint8 in host memory
and are scaled by 1/255 during the batch gather.  When the files are
missing it falls back, as the reference does (mnist.cpp:42-84), to a
synthetic set of U[0,1) images with uniform labels (1000 train / 200
test), here drawn from a seeded generator so runs are reproducible.
"""
from __future__ import annotations

import os

import torch

from .. import _ext
from .dataset import Dataset

IMAGE_SIZE = 28
NUM_CLASSES = 10


def read_idx(path: str) -> torch.Tensor:
    """Load an IDX file as a CPU tensor (u8 / i8 / i16 / i32 / f32 / f64)."""
    code, dims, raw = _ext.C().data.read_idx(path)
    dt = {0x08: torch.uint8, 0x09: torch.int8, 0x0B: torch.int16, 0x0C: torch.int32, 0x0D: torch.float32,
          0x0E: torch.float64}[code]
    t = torch.frombuffer(bytearray(raw), dtype=dt) if raw else torch.empty(0, dtype=dt)
    return t.reshape(dims).clone()


def write_idx(path: str, t: torch.Tensor) -> None:
    code = {torch.uint8: 0x08, torch.int8: 0x09, torch.int16: 0x0B, torch.int32: 0x0C, torch.float32: 0x0D,
            torch.float64: 0x0E}[t.dtype]
    _ext.C().data.write_idx(path, code, list(t.shape), t.contiguous().numpy().tobytes())


class MnistDataset(Dataset):
    IMAGE_SIZE = IMAGE_SIZE
    NUM_CLASSES = NUM_CLASSES

    def __init__(self, root: str, train: bool = True, download: bool = True, synthetic_seed: int = 0,
                 verbose: bool = False):
        self.root = root
        self.train = train
        prefix = "train" if train else "t10k"
        img = os.path.join(root, f"{prefix}-images-idx3-ubyte")
        lab = os.path.join(root, f"{prefix}-labels-idx1-ubyte")
        self.synthetic = not (os.path.exists(img) and os.path.exists(lab))
        if not self.synthetic:
            images = read_idx(img)
            labels = read_idx(lab)
            if images.dim() != 3 or labels.dim() != 1 or images.shape[0] != labels.shape[0]:
                raise ValueError("MNIST: image/label files do not match")
            self.images = images.reshape(images.shape[0], 1, images.shape[1], images.shape[2]).contiguous()
            self.labels = labels.to(torch.int32).contiguous()
            self._u8 = True
        else:
            # no network here, so `download` cannot fetch: synthetic fallback
            n = 1000 if train else 200
            g = torch.Generator().manual_seed(synthetic_seed + (0 if train else 1))
            self.images = torch.rand((n, 1, IMAGE_SIZE, IMAGE_SIZE), generator=g)
            self.labels = torch.randint(0, NUM_CLASSES, (n,), generator=g, dtype=torch.int32)
            self._u8 = False
            if verbose:
                print(f"MNIST files not found under {root}; synthetic {'train' if train else 'test'} set of {n}")

    def size(self) -> int:
        return int(self.images.shape[0])

    def get_item(self, index: int):
        x = self.images[index]
        x = x.float() / 255.0 if self._u8 else x.clone()
        return x, int(self.labels[index])

    def get_image_data(self, index: int) -> torch.Tensor:
        return self.get_item(index)[0].reshape(-1)

    def get_label(self, index: int) -> int:
        return int(self.labels[index])

    def input_shape(self):
        return [1, IMAGE_SIZE, IMAGE_SIZE]

    def target_shape(self):
        return [NUM_CLASSES]

    def num_classes(self) -> int:
        return NUM_CLASSES

    def arrays(self):
        return self.images, self.labels

    @property
    def u8_scale(self) -> float:
        return 1.0 / 255.0 if self._u8 else 1.0
