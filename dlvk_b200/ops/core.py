"""Op dispatch: CUDA tensors go to the hand-written sm_100a kernels in
`dlvk_b200._C`; CPU tensors take a plain PyTorch reference path with the same
semantics (used by the CPU test suite and as the oracle's twin).

There is no silent fallback for GPU tensors: if the native extension is
missing, every CUDA op raises.
"""
from __future__ import annotations

import torch

from .. import _ext

# Codes shared with csrc/include/dlvk/kernels.h
UN_RELU, UN_SIGMOID, UN_TANH, UN_SCALE, UN_CLAMP, UN_SQRT, UN_COPY = 0, 1, 2, 3, 4, 5, 6
UN_SQUARE, UN_ADD_SCALAR, UN_ABS, UN_EXP, UN_LOG, UN_GELU = 7, 8, 9, 10, 11, 12
BIN_ADD, BIN_SUB, BIN_MUL, BIN_DIV, BIN_MAX, BIN_MIN = 0, 1, 2, 3, 4, 5
BIN_RELU_BWD, BIN_SIGMOID_BWD, BIN_TANH_BWD, BIN_GELU_BWD = 6, 7, 8, 9
RED_SUM, RED_MAX, RED_MIN, RED_SUMSQ, RED_ABSMAX = 0, 1, 2, 3, 4
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2
OPT_SGD, OPT_ADAM, OPT_RMSPROP = 0, 1, 2
LOSS_MSE, LOSS_BCE = 0, 1

ACT_BY_NAME = {None: ACT_NONE, "none": ACT_NONE, "linear": ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU}


def N():
    """The native module (raises if it cannot be loaded)."""
    return _ext.C()


def native(t: torch.Tensor) -> bool:
    return t.is_cuda


# ---------------------------------------------------------------- activations
def _act_ref(x: torch.Tensor, act: int) -> torch.Tensor:
    if act == ACT_RELU:
        return torch.relu(x)
    if act == ACT_GELU:
        return torch.nn.functional.gelu(x)
    return x


def _unary_ref(x, op, a, b):
    xf = x.float()
    if op == UN_RELU:
        return torch.relu(xf)
    if op == UN_SIGMOID:
        return torch.sigmoid(xf)
    if op == UN_TANH:
        return torch.tanh(xf)
    if op == UN_SCALE:
        return xf * a
    if op == UN_CLAMP:
        return xf.clamp(a, b)
    if op == UN_SQRT:
        return xf.sqrt()
    if op == UN_COPY:
        return xf
    if op == UN_SQUARE:
        return xf * xf
    if op == UN_ADD_SCALAR:
        return xf + a
    if op == UN_ABS:
        return xf.abs()
    if op == UN_EXP:
        return xf.exp()
    if op == UN_LOG:
        return xf.log()
    if op == UN_GELU:
        return torch.nn.functional.gelu(xf)
    raise ValueError(op)


def unary(x: torch.Tensor, op: int, a: float = 0.0, b: float = 0.0, out_dtype=None) -> torch.Tensor:
    if native(x):
        return N().unary(x, op, a, b, out_dtype=out_dtype)
    return _unary_ref(x, op, a, b).to(out_dtype or x.dtype)


def _binary_ref(x, y, op):
    xf, yf = x.float(), y.float()
    if op == BIN_ADD:
        return xf + yf
    if op == BIN_SUB:
        return xf - yf
    if op == BIN_MUL:
        return xf * yf
    if op == BIN_DIV:
        guard = yf.abs() < 1e-8
        sign = torch.where(xf >= 0, torch.ones_like(xf), -torch.ones_like(xf))
        return torch.where(guard, sign * 1e8, xf / torch.where(guard, torch.ones_like(yf), yf))
    if op == BIN_MAX:
        return torch.maximum(xf, yf)
    if op == BIN_MIN:
        return torch.minimum(xf, yf)
    if op == BIN_RELU_BWD:
        return torch.where(yf > 0, xf, torch.zeros_like(xf))
    if op == BIN_SIGMOID_BWD:
        return xf * yf * (1 - yf)
    if op == BIN_TANH_BWD:
        return xf * (1 - yf * yf)
    if op == BIN_GELU_BWD:
        cdf = 0.5 * (1 + torch.erf(yf * 0.7071067811865476))
        pdf = 0.3989422804014327 * torch.exp(-0.5 * yf * yf)
        return xf * (cdf + yf * pdf)
    raise ValueError(op)


def binary(x: torch.Tensor, y: torch.Tensor, op: int) -> torch.Tensor:
    if native(x):
        if y.dtype != x.dtype:
            y = y.to(x.dtype)
        return N().binary(x, y, op)
    return _binary_ref(x, y, op).to(x.dtype)


def bias_act(x: torch.Tensor, bias, act_unary_op: int = UN_COPY) -> torch.Tensor:
    if native(x):
        return N().bias_act(x, bias, act_unary_op)
    y = x.float() + (bias.float() if bias is not None else 0.0)
    if act_unary_op != UN_COPY:
        y = _unary_ref(y, act_unary_op, 0.0, 0.0)
    return y.to(x.dtype)


# ---------------------------------------------------------------- reductions
def reduce(x: torch.Tensor, op: int = RED_SUM, scale: float = 1.0) -> torch.Tensor:
    if native(x):
        return N().reduce(x, op, scale)
    xf = x.float()
    r = {RED_SUM: xf.sum, RED_MAX: xf.max, RED_MIN: xf.min}.get(op)
    if r is not None:
        return r() * scale
    if op == RED_SUMSQ:
        return (xf * xf).sum() * scale
    if op == RED_ABSMAX:
        return xf.abs().max() * scale
    raise ValueError(op)


def colsum(x: torch.Tensor, scale: float = 1.0, out=None, accumulate: bool = False, out_dtype=None):
    if native(x):
        return N().colsum(x, scale, out=out, accumulate=accumulate, out_dtype=out_dtype)
    cols = x.shape[-1]
    s = x.reshape(-1, cols).float().sum(0) * scale
    if out is not None:
        if accumulate:
            out.add_(s.to(out.dtype))
        else:
            out.copy_(s)
        return out
    return s.to(out_dtype or torch.float32)


def transpose(x: torch.Tensor) -> torch.Tensor:
    if native(x):
        return N().transpose(x)
    return x.transpose(-1, -2).contiguous()


def permute4(x: torch.Tensor, perm) -> torch.Tensor:
    if native(x):
        return N().permute4(x, list(perm))
    return x.permute(*perm).contiguous()


# ---------------------------------------------------------------- GEMM
def relu_bits_like(m: int, n: int, device) -> torch.Tensor:
    """An int32 [m, ceil(n / 32)] buffer for a GEMM's ReLU bitmask."""
    return torch.empty(m, (n + 31) // 32, dtype=torch.int32, device=device)


def _pack_bits(pos: torch.Tensor, words: int) -> torch.Tensor:
    """[m, n] bool -> [m, words] int32, bit j of word w = pos[:, 32 w + j]."""
    m, n = pos.shape
    pad = torch.zeros(m, words * 32, dtype=torch.int64, device=pos.device)
    pad[:, :n] = pos.to(torch.int64)
    shifts = torch.arange(32, dtype=torch.int64, device=pos.device)
    w = (pad.reshape(m, words, 32) << shifts).sum(-1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _unpack_bits(bits: torch.Tensor, n: int) -> torch.Tensor:
    shifts = torch.arange(32, dtype=torch.int64, device=bits.device)
    b = (bits.to(torch.int64) & 0xFFFFFFFF).unsqueeze(-1) >> shifts
    return (b & 1).reshape(bits.shape[0], -1)[:, :n].bool()


def gemm(a: torch.Tensor, b: torch.Tensor, bias=None, act: int = ACT_NONE, alpha: float = 1.0, beta: float = 0.0,
         out=None, out_dtype=None, residual=None, relu_mask=None, colsum_out=None, colsum_scale: float = 1.0,
         colsum_accumulate: bool = False, relu_bits_out=None, relu_bits=None) -> torch.Tensor:
    """act(alpha * a @ b + beta * out + bias + residual), zeroed where
    relu_mask <= 0.  a: [M,K], [B,M,K] or [B,B2,M,K] (any strides), b
    likewise.  Transposes and head splits are views; the tensor-core path is
    used whenever the layout allows it.  With colsum_out (fp32 [N], 2-D
    GEMMs) the column sums of the result, times colsum_scale, are written
    (or added, colsum_accumulate) there as well: the bias gradient of a layer
    whose output gradient this GEMM produces.  relu_bits_out (int32
    [M, ceil(N / 32)], relu_bits_like) receives one bit per output element,
    set where the output is > 0; relu_bits zeroes the output where its bit is
    clear (2-D GEMMs): a ReLU's backward from 1/16 of a bf16 mask's bytes."""
    if native(a):
        return N().gemm(a, b, bias=bias, act=act, alpha=alpha, beta=beta, out=out, out_dtype=out_dtype,
                        residual=residual, relu_mask=relu_mask, colsum_out=colsum_out, colsum_scale=colsum_scale,
                        colsum_accumulate=colsum_accumulate, relu_bits_out=relu_bits_out, relu_bits=relu_bits)
    c = alpha * torch.matmul(a.float(), b.float())
    if beta != 0.0 and out is not None:
        c = c + beta * out.float()
    if bias is not None:
        c = c + bias.float()
    if residual is not None:
        c = c + residual.float()
    c = _act_ref(c, act)
    if relu_mask is not None:
        c = torch.where(relu_mask.float() > 0, c, torch.zeros_like(c))
    if relu_bits is not None:
        c = torch.where(_unpack_bits(relu_bits, c.shape[-1]), c, torch.zeros_like(c))
    if relu_bits_out is not None:
        relu_bits_out.copy_(_pack_bits(c > 0, relu_bits_out.shape[1]))
    if colsum_out is not None:
        s = c.reshape(-1, c.shape[-1]).sum(0) * colsum_scale
        if colsum_accumulate:
            colsum_out.add_(s)
        else:
            colsum_out.copy_(s)
    if out is not None:
        out.copy_(c)
        return out
    return c.to(out_dtype or a.dtype)


# ---------------------------------------------------------------- softmax / losses
def softmax(x: torch.Tensor, log: bool = False) -> torch.Tensor:
    if native(x):
        return N().softmax(x, log)
    xf = x.float()
    return (torch.log_softmax(xf, -1) if log else torch.softmax(xf, -1)).to(x.dtype)


def softmax_bwd(y: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    if native(y):
        return N().softmax_bwd(y, dy)
    yf, dyf = y.float(), dy.float()
    return (yf * (dyf - (yf * dyf).sum(-1, keepdim=True))).to(y.dtype)


def softmax_ce(logits: torch.Tensor, target: torch.Tensor, grad_scale: float = 1.0, want_grad: bool = True,
               in_place: bool = False):
    """Fused softmax + cross-entropy.  Returns (loss_rows f32 [rows], dlogits).
    target: int32 class ids (-1 = ignored row) or float probabilities."""
    if native(logits):
        if target.dtype not in (torch.int32,) and not target.is_floating_point():
            target = target.to(torch.int32)
        return tuple(N().softmax_ce(logits, target, grad_scale, want_grad, in_place))
    cols = logits.shape[-1]
    x = logits.reshape(-1, cols).float()
    lse = torch.logsumexp(x, -1)
    p = torch.softmax(x, -1)
    if not target.is_floating_point():
        lab = target.reshape(-1).long()
        valid = lab >= 0
        t = torch.zeros_like(x)
        t[valid, lab[valid]] = 1.0
        loss = torch.where(valid, lse - x.gather(1, lab.clamp(min=0)[:, None])[:, 0], torch.zeros_like(lse))
        g = (p - t) * grad_scale
        g[~valid] = 0
    else:
        t = target.reshape(-1, cols).float()
        loss = (t * (lse[:, None] - x)).sum(-1)
        g = (p - t) * grad_scale
    dl = None
    if want_grad:
        dl = g.to(logits.dtype).reshape(logits.shape)
        if in_place:
            logits.copy_(dl)
            dl = logits
    return loss, dl


def sum_scalar(v: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    if native(v):
        return N().sum_scalar(v, scale)
    return v.float().sum() * scale


def pointwise_loss(p: torch.Tensor, t: torch.Tensor, kind: int, loss_scale: float, grad_scale: float,
                   want_grad: bool = True):
    if native(p):
        return tuple(N().pointwise_loss(p, t, kind, loss_scale, grad_scale, want_grad))
    pf, tf = p.float(), t.float()
    if kind == LOSS_MSE:
        d = pf - tf
        loss = (d * d).sum() * loss_scale
        g = 2 * d * grad_scale
    else:
        pc = pf.clamp(1e-7, 1 - 1e-7)
        loss = (-(tf * pc.log() + (1 - tf) * (1 - pc).log())).sum() * loss_scale
        g = (pc - tf) / (pc * (1 - pc)) * grad_scale
    return loss, (g.to(p.dtype) if want_grad else None)
