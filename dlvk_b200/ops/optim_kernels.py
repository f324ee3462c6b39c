"""Device-resident optimizer hyper-parameter block (mirrors `OptimHyper` in
csrc/include/dlvk/kernels.h) and helpers to create and update it."""
from __future__ import annotations

import struct

import torch

# 10 floats, 4 ints, 2 pointers (clip coefficient, skip flag)
_FMT = "<10f4i2Q"
HYPER_BYTES = struct.calcsize(_FMT)
FIELDS = ("lr", "beta1", "beta2", "eps", "weight_decay", "momentum", "alpha", "grad_scale", "bc1", "bc2",
          "step", "bias_correction", "decoupled_wd", "pad_", "clip_coef_ptr", "skip_flag_ptr")


def pack_hyper(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0, momentum=0.0, alpha=0.99,
               grad_scale=1.0, step=0, bias_correction=True, decoupled_wd=False, clip_coef_ptr=0,
               skip_flag_ptr=0) -> bytes:
    return struct.pack(_FMT, lr, beta1, beta2, eps, weight_decay, momentum, alpha, grad_scale, 1.0, 1.0,
                       int(step), int(bool(bias_correction)), int(bool(decoupled_wd)), 0, int(clip_coef_ptr),
                       int(skip_flag_ptr))


def make_hyper(device, **kw) -> torch.Tensor:
    """Allocate the hyper block on `device` as a uint8 tensor."""
    raw = bytearray(pack_hyper(**kw))
    t = torch.frombuffer(raw, dtype=torch.uint8).clone()
    return t.to(device) if torch.device(device).type == "cuda" else t


def read_hyper(t: torch.Tensor) -> dict:
    vals = struct.unpack(_FMT, bytes(t.detach().cpu().numpy().tobytes()))
    return dict(zip(FIELDS, vals))


def _field_code(idx: int) -> str:
    if idx < 10:
        return "f"
    if idx < 14:
        return "i"
    return "Q"


def field_offset(name: str) -> int:
    idx = FIELDS.index(name)
    return 4 * idx if idx < 14 else 56 + 8 * (idx - 14)


def set_field(t: torch.Tensor, name: str, value) -> None:
    idx = FIELDS.index(name)
    code = _field_code(idx)
    b = struct.pack("<" + code, value)
    off = field_offset(name)
    src = torch.frombuffer(bytearray(b), dtype=torch.uint8)
    t[off:off + len(b)].copy_(src)
