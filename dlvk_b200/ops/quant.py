"""int8 quantisation ops (native kernels on GPU, integer-exact PyTorch
reference on CPU)."""
from __future__ import annotations

import torch

from .core import N, native, ACT_NONE, ACT_RELU


def quantize_rows(x: torch.Tensor):
    """Symmetric per-row int8: returns (q int8 [rows, cols], scale f32 [rows])."""
    x2 = x.reshape(-1, x.shape[-1])
    if native(x2):
        q, s = N().quantize_rows(x2)
        return q, s
    xf = x2.float()
    mx = xf.abs().amax(-1)
    s = torch.where(mx > 0, mx / 127.0, torch.ones_like(mx))
    q = torch.round(xf / s[:, None]).clamp(-127, 127).to(torch.int8)
    return q, s


def gemm_i8(qa, qbt, sa, sb, bias=None, act: int = ACT_NONE, out_dtype=torch.float32):
    """act(qa @ qbt^T * sa[:, None] * sb[None, :] + bias) with int32 accumulation."""
    if native(qa):
        return N().gemm_i8(qa, qbt, sa, sb, bias, act, out_dtype)
    acc = qa.to(torch.int64) @ qbt.to(torch.int64).t()
    y = acc.to(torch.float64) * sa.double()[:, None] * sb.double()[None, :]
    if bias is not None:
        y = y + bias.double()
    if act == ACT_RELU:
        y = torch.relu(y)
    return y.to(out_dtype)
