"""The benchmark models written in plain PyTorch (cuBLAS / cuDNN / SDPA
kernels, torch optimizers, NCCL via DDP): the comparison point for the
framework's own kernels.  Same shapes, same optimizers, same dtypes."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..models import zoo


class Block(nn.Module):
    def __init__(self, d, h, ff):
        super().__init__()
        self.h = h
        self.ln1 = nn.LayerNorm(d)
        self.qkv = nn.Linear(d, 3 * d, bias=False)
        self.o = nn.Linear(d, d, bias=False)
        self.ln2 = nn.LayerNorm(d)
        self.f1 = nn.Linear(d, ff)
        self.f2 = nn.Linear(ff, d)

    def forward(self, x):
        B, S, D = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(B, S, 3, self.h, D // self.h).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, S, D)
        x = x + self.o(a)
        return x + self.f2(F.relu(self.f1(self.ln2(x))))


class TorchTransformer(nn.Module):
    def __init__(self, vocab=32000, d=1024, layers=12, h=16, ff=4096):
        super().__init__()
        self.emb = nn.Embedding(vocab, d)
        self.blocks = nn.ModuleList([Block(d, h, ff) for _ in range(layers)])
        self.ln = nn.LayerNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)
        for p in self.parameters():
            if p.dim() > 1:
                nn.init.normal_(p, 0.0, 0.02)

    def forward(self, ids):
        x = self.emb(ids)
        for b in self.blocks:
            x = b(x)
        return self.head(self.ln(x))


def wide_mlp():
    layers = [nn.Linear(1024, 4096)]
    for _ in range(4):
        layers += [nn.Linear(4096, 4096), nn.BatchNorm1d(4096), nn.ReLU(), nn.Dropout(0.1)]
    layers += [nn.Linear(4096, 1000)]
    return nn.Sequential(*layers)


def cnn():
    return nn.Sequential(nn.Conv2d(1, 8, 3, 1, 1), nn.ReLU(), nn.MaxPool2d(2), nn.Conv2d(8, 16, 3, 1, 1), nn.ReLU(),
                         nn.MaxPool2d(2), nn.Flatten(), nn.Linear(784, 128), nn.ReLU(), nn.Linear(128, 47))


def mlp():
    return nn.Sequential(nn.Linear(784, 128), nn.ReLU(), nn.Linear(128, 10))


def build_torch(name: str, local: int, rank: int):
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    zc = zoo.CONFIGS[name]
    base = "cnn" if name.startswith("cnn") else name
    model = {"transformer": TorchTransformer, "wide_mlp": wide_mlp, "cnn": cnn, "mlp": mlp}[base]().to(dev)
    if zc.optimizer == "adam":
        # capturable: the step counter stays on the device, so the whole
        # training step can be captured into a CUDA graph
        opt = torch.optim.Adam(model.parameters(), lr=1e-3, fused=True, capturable=True)
    else:
        opt = torch.optim.SGD(model.parameters(), lr=0.01, momentum=0.9, foreach=True)
    x, y = zoo.synthetic_batch(base, zc.batch, seed=1000 + rank, seq_len=zc.seq_len or 512)
    if base == "transformer":
        x = x.long()
    xd, yd = x.to(dev), y.to(dev)
    return model, opt, zc.batch, zc.seq_len, zc.dtype, (lambda: (xd, yd))
