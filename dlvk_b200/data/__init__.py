"""Data subsystem: datasets, MNIST, the prefetching DataLoader and
batched device transforms (include/dlvk/data/*)."""
from .dataset import Dataset, SyntheticDataset, TensorDataset, TransformDataset
from .mnist import MnistDataset, read_idx, write_idx
from .dataloader import DataLoader
from . import transforms

__all__ = ["Dataset", "SyntheticDataset", "TensorDataset", "TransformDataset", "MnistDataset", "read_idx",
           "write_idx", "DataLoader", "transforms"]
