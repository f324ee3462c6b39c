"""Layer-level ops (convolution, pooling, norms, dropout, embedding,
attention) with native CUDA paths and plain-PyTorch CPU reference paths."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .core import N, native, gemm, softmax, softmax_bwd, ACT_NONE


# ---------------------------------------------------------------- convolution
def conv2d_fwd(x, w, bias, stride: int, pad: int, relu: bool = False):
    if native(x):
        return N().conv2d_fwd(x, w, bias, stride, pad, relu)
    y = F.conv2d(x.float(), w.float(), bias.float() if bias is not None else None, stride=stride, padding=pad)
    if relu:
        y = torch.relu(y)
    return y.to(x.dtype)


def conv2d_dgrad(gy, w, xshape, stride: int, pad: int, relu_src=None):
    if native(gy):
        return N().conv2d_dgrad(gy, w, list(xshape), stride, pad, relu_src)
    dx = torch.nn.grad.conv2d_input(list(xshape), w.float(), gy.float(), stride=stride, padding=pad)
    if relu_src is not None:
        dx = torch.where(relu_src.float() > 0, dx, torch.zeros_like(dx))
    return dx.to(gy.dtype)


def conv2d_wgrad(x, gy, dw, db, stride: int, pad: int, accumulate: bool = False):
    if native(x):
        N().conv2d_wgrad(x, gy, dw, db, stride, pad, accumulate)
        return
    gw = torch.nn.grad.conv2d_weight(x.float(), list(dw.shape), gy.float(), stride=stride, padding=pad)
    gb = gy.float().sum((0, 2, 3))
    if accumulate:
        dw.add_(gw)
        if db is not None:
            db.add_(gb)
    else:
        dw.copy_(gw)
        if db is not None:
            db.copy_(gb)


# ---------------------------------------------------------------- pooling
def maxpool_fwd(x, k: int, stride: int):
    if native(x):
        y, idx = N().maxpool_fwd(x, k, stride)
        return y, idx
    Nn, C, H, W = x.shape
    y, idx = F.max_pool2d(x.float(), k, stride, return_indices=True)
    return y.to(x.dtype), idx.to(torch.int32)


def maxpool_bwd(gy, idx, H: int, W: int, k: int, stride: int):
    if native(gy):
        return N().maxpool_bwd(gy, idx, H, W, k, stride)
    Nn, C = gy.shape[:2]
    dx = torch.zeros(Nn, C, H * W, dtype=torch.float32)
    dx.scatter_add_(2, idx.reshape(Nn, C, -1).long(), gy.float().reshape(Nn, C, -1))
    return dx.reshape(Nn, C, H, W).to(gy.dtype)


def avgpool_fwd(x, k: int, stride: int, pad: int = 0):
    if native(x):
        return N().avgpool_fwd(x, k, stride, pad)
    return F.avg_pool2d(x.float(), k, stride, pad, count_include_pad=False).to(x.dtype)


def avgpool_bwd(gy, H: int, W: int, k: int, stride: int, pad: int = 0):
    if native(gy):
        return N().avgpool_bwd(gy, H, W, k, stride, pad)
    x = torch.zeros(gy.shape[0], gy.shape[1], H, W, requires_grad=True)
    with torch.enable_grad():
        y = F.avg_pool2d(x, k, stride, pad, count_include_pad=False)
        (dx,) = torch.autograd.grad(y, x, gy.float())
    return dx.to(gy.dtype)


# ---------------------------------------------------------------- dropout masks (CPU twin of the kernels)
def philox_keep_mask(numel: int, p: float, seed: int, stream: int, step: int) -> torch.Tensor:
    """Keep mask identical to the CUDA kernels' Philox stream (CPU, via the C++ oracle)."""
    return N().ref.dropout_mask(int(numel), float(p), int(seed), int(stream), int(step)).bool()


def _cpu_step(step, step_t):
    return int(step_t.item()) if step_t is not None else int(step)


# ---------------------------------------------------------------- batch norm (+relu +dropout)
def batchnorm_fwd(x, gamma, beta, run_mean, run_var, momentum: float, eps: float, training: bool,
                  relu: bool = False, p: float = 0.0, stream: int = 0, seed: int = 0, step: int = 0, step_t=None):
    if native(x):
        return tuple(N().batchnorm_fwd(x, gamma, beta, run_mean, run_var, momentum, eps, training, relu, p, stream,
                                       seed, step, step_t))
    C = x.shape[1]
    xf = x.float()
    dims = [0] + list(range(2, x.dim()))
    shape = [1, C] + [1] * (x.dim() - 2)
    if training:
        mean = xf.mean(dims)
        var = xf.var(dims, unbiased=False)
        if run_mean is not None:
            run_mean.mul_(1 - momentum).add_(momentum * mean)
            run_var.mul_(1 - momentum).add_(momentum * var)
    else:
        mean, var = run_mean.float(), run_var.float()
    rstd = torch.rsqrt(var + eps)
    y = (xf - mean.reshape(shape)) * rstd.reshape(shape)
    if gamma is not None:
        y = y * gamma.reshape(shape) + beta.reshape(shape)
    if relu:
        y = torch.relu(y)
    if training and p > 0:
        keep = philox_keep_mask(y.numel(), p, seed, stream, _cpu_step(step, step_t)).reshape(y.shape)
        y = torch.where(keep, y / (1 - p), torch.zeros_like(y))
    return y.to(x.dtype), mean, rstd


def batchnorm_bwd(x, dy, mean, rstd, gamma, beta, dgamma, dbeta, accumulate: bool, relu: bool = False,
                  p: float = 0.0, stream: int = 0, seed: int = 0, step: int = 0, step_t=None):
    if native(x):
        return N().batchnorm_bwd(x, dy, mean, rstd, gamma, beta, dgamma, dbeta, accumulate, relu, p, stream, seed,
                                 step, step_t)
    C = x.shape[1]
    dims = [0] + list(range(2, x.dim()))
    shape = [1, C] + [1] * (x.dim() - 2)
    xh = (x.float() - mean.reshape(shape)) * rstd.reshape(shape)
    g = dy.float()
    if p > 0:
        keep = philox_keep_mask(g.numel(), p, seed, stream, _cpu_step(step, step_t)).reshape(g.shape)
        g = torch.where(keep, g / (1 - p), torch.zeros_like(g))
    gm = gamma.reshape(shape) if gamma is not None else 1.0
    if relu:
        pre = xh * gm + (beta.reshape(shape) if beta is not None else 0.0)
        g = torch.where(pre > 0, g, torch.zeros_like(g))
    sg = g.sum(dims)
    sgx = (g * xh).sum(dims)
    cnt = x.numel() // C
    dx = gm * rstd.reshape(shape) * (g - sg.reshape(shape) / cnt - xh * sgx.reshape(shape) / cnt)
    for buf, val in ((dgamma, sgx), (dbeta, sg)):
        if buf is not None:
            buf.add_(val) if accumulate else buf.copy_(val)
    return dx.to(x.dtype)


# ---------------------------------------------------------------- layer norm
def layernorm_fwd(x, gamma, beta, eps: float):
    if native(x):
        return tuple(N().layernorm_fwd(x, gamma, beta, eps))
    xf = x.float()
    mean = xf.mean(-1)
    var = xf.var(-1, unbiased=False)
    rstd = torch.rsqrt(var + eps)
    y = (xf - mean[..., None]) * rstd[..., None]
    if gamma is not None:
        y = y * gamma + beta
    D = x.shape[-1]
    return y.to(x.dtype), mean.reshape(-1), rstd.reshape(-1)


def layernorm_bwd(x, gamma, mean, rstd, dy, dgamma, dbeta, accumulate: bool, dres=None, dres_colsum=None,
                  dres_colsum_accumulate: bool = False):
    """dx (+ dres, the gradient of a residual branch sharing the input).
    dres_colsum (fp32 [D]) receives, or with dres_colsum_accumulate adds, the
    column sums of dres: the bias gradient of the biased GEMM whose output
    gradient dres is, taken in the same pass."""
    if native(x):
        return N().layernorm_bwd(x, gamma, mean, rstd, dy, dgamma, dbeta, accumulate, dres,
                                 dres_colsum=dres_colsum, dres_colsum_accumulate=dres_colsum_accumulate)
    if dres is not None:
        if dres_colsum is not None:
            cs = dres.float().reshape(-1, dres.shape[-1]).sum(0)
            dres_colsum.add_(cs) if dres_colsum_accumulate else dres_colsum.copy_(cs)
        out = layernorm_bwd(x, gamma, mean, rstd, dy, dgamma, dbeta, accumulate)
        return (out.float() + dres.float()).to(x.dtype)
    D = x.shape[-1]
    xf = x.float().reshape(-1, D)
    g = dy.float().reshape(-1, D)
    xh = (xf - mean[:, None]) * rstd[:, None]
    gg = g * (gamma if gamma is not None else 1.0)
    a = gg.mean(-1, keepdim=True)
    b = (gg * xh).mean(-1, keepdim=True)
    dx = rstd[:, None] * (gg - a - xh * b)
    for buf, val in ((dgamma, (g * xh).sum(0)), (dbeta, g.sum(0))):
        if buf is not None:
            buf.add_(val) if accumulate else buf.copy_(val)
    return dx.reshape(x.shape).to(x.dtype)


# ---------------------------------------------------------------- dropout
def dropout(x, p: float, stream: int, seed: int, step: int = 0, step_t=None):
    if native(x):
        return N().dropout(x, p, stream, seed, step, step_t)
    keep = philox_keep_mask(x.numel(), p, seed, stream, _cpu_step(step, step_t)).reshape(x.shape)
    return torch.where(keep, x.float() / (1 - p), torch.zeros_like(x, dtype=torch.float32)).to(x.dtype)


# ---------------------------------------------------------------- embedding
def embedding_fwd(ids, table):
    if native(table):
        return N().embedding_fwd(ids.to(torch.int32), table)
    idl = ids.long()
    ok = (idl >= 0) & (idl < table.shape[0])
    out = table[idl.clamp(0, table.shape[0] - 1)]
    return torch.where(ok[..., None], out, torch.zeros_like(out))


def embedding_bwd(ids, dy, dtable):
    """Accumulates into dtable (caller zeroes it)."""
    if native(dy):
        N().embedding_bwd(ids.to(torch.int32), dy, dtable)
        return
    idl = ids.reshape(-1).long()
    ok = (idl >= 0) & (idl < dtable.shape[0])
    dtable.index_add_(0, idl[ok], dy.reshape(-1, dtable.shape[1]).float()[ok])


# ---------------------------------------------------------------- attention
def flash_ok(qkv, B: int, S: int, H: int, D: int) -> bool:
    """The fused tcgen05 attention kernels apply: bf16, head dim 64, S a
    multiple of 128 (DLVK_FLASH_ATTN=0 disables them)."""
    import os

    return (native(qkv) and qkv.dtype == torch.bfloat16 and os.environ.get("DLVK_FLASH_ATTN", "1") != "0"
            and N().flash_attn_supported(B, S, H, D, qkv))


def attention_fwd(qkv, B: int, S: int, H: int, D: int, scale: float):
    """Multi-head attention over a fused QKV buffer [B, S, 3, H, D] (the QKV
    GEMM's natural output).  Returns (out [B, S, H*D], aux) where aux is the
    per-row log-sum-exp [B, H, S] (fp32, log2 units) on the fused tensor-core
    path, or the probabilities [B, H, S, S] on the GEMM + softmax path."""
    E = H * D
    if flash_ok(qkv, B, S, H, D):
        return N().flash_attn_fwd(qkv.contiguous(), B, S, H, scale)
    if native(qkv):
        base = qkv.reshape(-1)
        o0 = base.storage_offset()
        q = base.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), o0)
        k = base.as_strided((B, H, D, S), (S * 3 * E, D, 1, 3 * E), o0 + E)
        v = base.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), o0 + 2 * E)
        scores = gemm(q, k, alpha=scale)                     # [B,H,S,S] (bf16 or f32)
        probs = softmax(scores)
        out = torch.empty(B, S, E, dtype=qkv.dtype, device=qkv.device)
        ov = out.as_strided((B, H, S, D), (S * E, D, E, 1), 0)
        gemm(probs, v, out=ov)
        return out, probs
    x = qkv.float().reshape(B, S, 3, H, D)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    sc = torch.matmul(q, k.transpose(-1, -2)) * scale
    probs = torch.softmax(sc, -1).to(qkv.dtype)
    o = torch.matmul(probs.float(), v)
    return o.transpose(1, 2).reshape(B, S, E).to(qkv.dtype), probs


def attention_bwd(qkv, probs, dout, B: int, S: int, H: int, D: int, scale: float, out=None):
    """Gradient of attention_fwd w.r.t. the fused QKV buffer: [B, S, 3*H*D].
    `probs` is attention_fwd's aux output; the fused path (aux = lse) also
    needs the forward output `out`."""
    E = H * D
    if probs.dim() == 3 and probs.dtype == torch.float32 and native(qkv):
        if out is None:
            raise ValueError("attention_bwd on the fused path needs the forward output")
        return N().flash_attn_bwd(qkv.contiguous(), out.reshape(B, S, E).contiguous(),
                                  dout.reshape(B, S, E).contiguous(), probs, B, S, H, scale)
    if native(qkv):
        base = qkv.reshape(-1)
        o0 = base.storage_offset()
        q = base.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), o0)
        k = base.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), o0 + E)
        vT = base.as_strided((B, H, D, S), (S * 3 * E, D, 1, 3 * E), o0 + 2 * E)
        dflat = dout.contiguous().reshape(-1)
        do = dflat.as_strided((B, H, S, D), (S * E, D, E, 1), dflat.storage_offset())
        dqkv = torch.empty(B, S, 3 * E, dtype=qkv.dtype, device=qkv.device)
        db = dqkv.reshape(-1)
        dq = db.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), 0)
        dk = db.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), E)
        dv = db.as_strided((B, H, S, D), (S * 3 * E, D, 3 * E, 1), 2 * E)
        pT = probs.transpose(-1, -2)
        gemm(pT, do, out=dv)                                   # dV = P^T dO
        dp = gemm(do, vT)                                      # dP = dO V^T
        ds = softmax_bwd(probs, dp)                            # dS = P (dP - rowsum(dP P))
        gemm(ds, k, alpha=scale, out=dq)                       # dQ = scale dS K
        gemm(ds.transpose(-1, -2), q, alpha=scale, out=dk)     # dK = scale dS^T Q
        return dqkv
    x = qkv.float().reshape(B, S, 3, H, D)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    p = probs.float()
    do = dout.float().reshape(B, S, H, D).transpose(1, 2)
    dv = torch.matmul(p.transpose(-1, -2), do)
    dp = torch.matmul(do, v.transpose(-1, -2))
    ds = p * (dp - (dp * p).sum(-1, keepdim=True))
    dq = torch.matmul(ds, k) * scale
    dk = torch.matmul(ds.transpose(-1, -2), q) * scale
    out = torch.stack([dq, dk, dv], dim=2)  # [B,H,3,S,D]
    return out.permute(0, 3, 2, 1, 4).reshape(B, S, 3 * E).to(qkv.dtype)
