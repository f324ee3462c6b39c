"""The benchmark model configurations, built from the public layer API.

  mlp          Dense 784->128, ReLU, Dense 128->10, Softmax (fp32)
  cnn          Conv2D 1->8 3x3 p1, ReLU, MaxPool 2, Conv2D 8->16 3x3 p1, ReLU,
               MaxPool 2, flatten 784, Dense 784->128, ReLU, Dense 128->47,
               Softmax
  wide_mlp     input Dense 1024->4096, then 4 x [Dense 4096->4096,
               BatchNorm1D, ReLU, Dropout(0.1)], output Dense 4096->1000,
               Softmax: the layer list exactly as the workload states it
               (only the 4096->4096 layers carry BatchNorm / ReLU / Dropout).
               It has 75.5M parameters; the workload's "~54M" does not match
               its own layer list.
  transformer  Embedding 32000 x 1024, 12 pre-norm encoder blocks (LayerNorm,
               16-head attention, LayerNorm, Dense 1024->4096, ReLU,
               Dense 4096->1024, residual adds), final LayerNorm and an
               untied Dense 1024->32000 head for next-token cross-entropy;
               weights N(0, 0.02).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .sequential import Sequential
from . import layers as L


@dataclass
class ZooConfig:
    name: str
    batch: int          # per GPU
    dtype: str
    optimizer: str
    seq_len: int = 0


CONFIGS = {
    "mlp": ZooConfig("mlp", 32, "fp32", "adam"),
    "cnn": ZooConfig("cnn", 256, "fp32", "adam"),
    "cnn_bf16": ZooConfig("cnn_bf16", 256, "bf16", "adam"),
    "wide_mlp": ZooConfig("wide_mlp", 1024, "bf16", "sgd"),
    "transformer": ZooConfig("transformer", 16, "bf16", "adam", seq_len=512),
}


def mlp(device=None, dtype="fp32", seed=0) -> Sequential:
    m = Sequential(device, dtype, seed=seed)
    m.add_dense(784, 128)
    m.add_relu()
    m.add_dense(128, 10)
    m.add_softmax()
    return m


def small_cnn(device=None, dtype="fp32", seed=0, num_classes=47) -> Sequential:
    m = Sequential(device, dtype, seed=seed)
    m.add_conv2d(1, 8, 3, 1, 1)
    m.add_relu()
    m.add_maxpool2d(2, 2)
    m.add_conv2d(8, 16, 3, 1, 1)
    m.add_relu()
    m.add_maxpool2d(2, 2)
    m.add_flatten()
    m.add_dense(784, 128)
    m.add_relu()
    m.add_dense(128, num_classes)
    m.add_softmax()
    return m


def wide_mlp(device=None, dtype="bf16", seed=0, width=4096, depth=4, d_in=1024, n_out=1000, p=0.1) -> Sequential:
    m = Sequential(device, dtype, seed=seed)
    m.add_dense(d_in, width)
    for _ in range(depth):
        m.add_dense(width, width)
        m.add_batchnorm1d(width)
        m.add_relu()
        m.add_dropout(p)
    m.add_dense(width, n_out)
    m.add_softmax()
    return m


def transformer(device=None, dtype="bf16", seed=0, vocab=32000, d_model=1024, layers=12, heads=16, d_ff=4096,
                std=0.02) -> Sequential:
    m = Sequential(device, dtype, seed=seed)
    m.add_embedding(vocab, d_model, init_std=std)
    for _ in range(layers):
        m.add_transformer_encoder(d_model, heads, d_ff, init_std=std)
    m.add_layernorm(d_model)
    m.add_dense(d_model, vocab, use_bias=False, init_std=std)
    m.add_softmax()
    return m


def build(name: str, device=None, seed=0, **kw) -> Sequential:
    cfg = CONFIGS[name]
    if name == "mlp":
        return mlp(device, kw.get("dtype", cfg.dtype), seed)
    if name.startswith("cnn"):
        return small_cnn(device, kw.get("dtype", cfg.dtype), seed)
    if name == "wide_mlp":
        return wide_mlp(device, kw.get("dtype", cfg.dtype), seed)
    if name == "transformer":
        return transformer(device, kw.get("dtype", cfg.dtype), seed, **{k: v for k, v in kw.items() if k != "dtype"})
    raise KeyError(name)


def synthetic_batch(name: str, batch: int, device="cpu", seed=0, seq_len: int = 512, vocab: int = 32000):
    """Synthetic inputs of the configuration's shapes (x, labels)."""
    g = torch.Generator().manual_seed(seed)
    if name == "mlp":
        return torch.rand(batch, 784, generator=g), torch.randint(0, 10, (batch,), generator=g, dtype=torch.int32)
    if name.startswith("cnn"):
        return (torch.rand(batch, 1, 28, 28, generator=g),
                torch.randint(0, 47, (batch,), generator=g, dtype=torch.int32))
    if name == "wide_mlp":
        return torch.randn(batch, 1024, generator=g), torch.randint(0, 1000, (batch,), generator=g, dtype=torch.int32)
    if name == "transformer":
        toks = torch.randint(0, vocab, (batch, seq_len + 1), generator=g, dtype=torch.int32)
        return toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    raise KeyError(name)
