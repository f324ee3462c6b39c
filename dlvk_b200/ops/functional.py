"""Autograd functions over the native kernels.

Parameters are not autograd leaves: each function writes dW/db straight into
the parameter's slice of the flat gradient buffer (overwriting on the first
write after ``zero_grad``, accumulating afterwards) and then fires the
parameter's grad-ready hooks, which the data-parallel bucketer uses to start
the fused all-reduce + optimizer of a bucket while backward continues.
Autograd only tracks activations.
"""
from __future__ import annotations

import math
import os

import torch

from . import core as K
from . import nn as NN
from .core import ACT_NONE, ACT_RELU, ACT_GELU

# DLVK_FUSE_COLSUM=0: bias gradients by a separate column-sum pass instead of
# the producing GEMM's epilogue.
_FUSE_COLSUM = os.environ.get("DLVK_FUSE_COLSUM", "1") != "0"
# The FFN's ReLU backward from a bitmask written by the forward GEMM (1), or
# from the bf16 activation itself (0).
_RELU_BITS = os.environ.get("DLVK_RELU_BITS", "1") != "0"


def _flat2(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1])


# Parameters are not autograd leaves, so every parametric function also takes
# this grad-requiring anchor: it makes the op's output part of the autograd
# graph even when the input activation does not require grad (first layer).
_ANCHOR = torch.zeros((), requires_grad=True)


def zero_(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        K.N().memset_zero(t)
    else:
        t.zero_()
    return t


class DenseFn(torch.autograd.Function):
    """y = act(x @ W + b [+ residual]); W stored [in, out] (reference layout,
    src/layers/dense_layer.cpp:16-20).

    fuse flags (set by the model's execution plan):
      mask_input  x is the output of a ReLU consumed only here: the dX GEMM
                  epilogue applies that ReLU's backward (zero where x <= 0);
      defer_relu  this op's own ReLU backward is applied by its consumer.
    """

    @staticmethod
    def forward(ctx, x, residual, anchor, W, b, act, mask_input=False, defer_relu=False):
        x2 = _flat2(x)
        r2 = _flat2(residual) if residual is not None else None
        y = K.gemm(x2, W.value, bias=b.master if b is not None else None, act=act, residual=r2)
        ctx.W, ctx.b, ctx.act = W, b, act
        ctx.has_res = residual is not None
        ctx.mask_input = mask_input
        ctx.relu_here = act == ACT_RELU and not defer_relu
        if act == ACT_GELU:
            raise NotImplementedError("GELU is not fused into the dense GEMM")
        ctx.save_for_backward(x2, y if ctx.relu_here else None)
        return y.reshape(*x.shape[:-1], W.shape[1])

    @staticmethod
    def backward(ctx, gy):
        x2, saved = ctx.saved_tensors
        W, b = ctx.W, ctx.b
        g2 = _flat2(gy)
        if g2.dtype != x2.dtype:
            g2 = g2.to(x2.dtype)
        if ctx.relu_here:
            g2 = K.binary(g2.contiguous(), saved, K.BIN_RELU_BWD)
        acc = W.take_accumulate_flag()
        K.gemm(x2.t(), g2, out=W.grad, beta=1.0 if acc else 0.0)
        if b is not None:
            K.colsum(g2, out=b.grad, accumulate=b.take_accumulate_flag())
        dx = None
        if ctx.needs_input_grad[0]:
            dx = K.gemm(g2, W.value.t(), relu_mask=x2 if ctx.mask_input else None).reshape(*gy.shape[:-1],
                                                                                          W.shape[0])
        # Hooks fire only after the last read of W in this backward: a
        # data-parallel bucket may update W in place as soon as it is ready.
        W.grad_ready()
        if b is not None:
            b.grad_ready()
        dres = gy if ctx.has_res and ctx.needs_input_grad[1] else None
        return dx, dres, None, None, None, None, None, None


def dense(x, W, b=None, act=ACT_NONE, residual=None, mask_input=False, defer_relu=False):
    return DenseFn.apply(x, residual, _ANCHOR, W, b, act, mask_input, defer_relu)


class ActivationFn(torch.autograd.Function):
    """relu / sigmoid / tanh / gelu with the saved tensor the backward needs
    (the reference passed zero dummies, src/layers/activation.cpp:51-69)."""

    _FWD = {"relu": K.UN_RELU, "sigmoid": K.UN_SIGMOID, "tanh": K.UN_TANH, "gelu": K.UN_GELU}
    _BWD = {"relu": K.BIN_RELU_BWD, "sigmoid": K.BIN_SIGMOID_BWD, "tanh": K.BIN_TANH_BWD, "gelu": K.BIN_GELU_BWD}

    @staticmethod
    def forward(ctx, x, kind):
        y = K.unary(x, ActivationFn._FWD[kind])
        ctx.kind = kind
        ctx.save_for_backward(x if kind == "gelu" else y)
        return y

    @staticmethod
    def backward(ctx, gy):
        (s,) = ctx.saved_tensors
        return K.binary(gy.contiguous(), s, ActivationFn._BWD[ctx.kind]), None


class SoftmaxFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = K.softmax(x)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, gy):
        (y,) = ctx.saved_tensors
        return K.softmax_bwd(y, gy.contiguous())


class Conv2dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, anchor, W, b, stride, pad, relu):
        y = NN.conv2d_fwd(x.contiguous(), W.value, b.master if b is not None else None, stride, pad, relu)
        ctx.W, ctx.b, ctx.stride, ctx.pad, ctx.relu = W, b, stride, pad, relu
        ctx.xshape = tuple(x.shape)
        ctx.save_for_backward(x, y if relu else None)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, y = ctx.saved_tensors
        g = gy.contiguous()
        if g.dtype != x.dtype:
            g = g.to(x.dtype)
        if ctx.relu:
            g = K.binary(g, y, K.BIN_RELU_BWD)
        W, b = ctx.W, ctx.b
        acc = W.take_accumulate_flag()
        if b is not None:
            b.take_accumulate_flag()
        NN.conv2d_wgrad(x, g, W.grad, b.grad if b is not None else None, ctx.stride, ctx.pad, accumulate=acc)
        dx = NN.conv2d_dgrad(g, W.value, ctx.xshape, ctx.stride, ctx.pad) if ctx.needs_input_grad[0] else None
        W.grad_ready()
        if b is not None:
            b.grad_ready()
        return dx, None, None, None, None, None, None


class MaxPoolFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, k, stride):
        y, idx = NN.maxpool_fwd(x.contiguous(), k, stride)
        ctx.k, ctx.stride, ctx.hw = k, stride, (x.shape[2], x.shape[3])
        ctx.save_for_backward(idx)
        return y

    @staticmethod
    def backward(ctx, gy):
        (idx,) = ctx.saved_tensors
        return NN.maxpool_bwd(gy.contiguous(), idx, ctx.hw[0], ctx.hw[1], ctx.k, ctx.stride), None, None


class AvgPoolFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, k, stride, pad):
        ctx.k, ctx.stride, ctx.pad, ctx.hw = k, stride, pad, (x.shape[2], x.shape[3])
        return NN.avgpool_fwd(x.contiguous(), k, stride, pad)

    @staticmethod
    def backward(ctx, gy):
        return NN.avgpool_bwd(gy.contiguous(), ctx.hw[0], ctx.hw[1], ctx.k, ctx.stride, ctx.pad), None, None, None


class BatchNormFn(torch.autograd.Function):
    """Batch norm with optional fused ReLU and Philox dropout after it."""

    @staticmethod
    def forward(ctx, x, anchor, gamma, beta, run_mean, run_var, cfg):
        y, mean, rstd = NN.batchnorm_fwd(x.contiguous(), gamma.master if gamma else None,
                                         beta.master if beta else None, run_mean, run_var, cfg["momentum"],
                                         cfg["eps"], cfg["training"], cfg["relu"], cfg["p"], cfg["stream"],
                                         cfg["seed"], 0, cfg["step_t"])
        ctx.gamma, ctx.beta, ctx.cfg = gamma, beta, cfg
        ctx.save_for_backward(x, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, mean, rstd = ctx.saved_tensors
        gamma, beta, cfg = ctx.gamma, ctx.beta, ctx.cfg
        acc = gamma.take_accumulate_flag() if gamma is not None else False
        if beta is not None:
            beta.take_accumulate_flag()
        dx = NN.batchnorm_bwd(x.contiguous(), gy.contiguous().to(x.dtype), mean, rstd,
                              gamma.master if gamma else None, beta.master if beta else None,
                              gamma.grad if gamma else None, beta.grad if beta else None, acc, cfg["relu"],
                              cfg["p"] if cfg["training"] else 0.0, cfg["stream"], cfg["seed"], 0, cfg["step_t"])
        if gamma is not None:
            gamma.grad_ready()
        if beta is not None:
            beta.grad_ready()
        return dx, None, None, None, None, None, None


class LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, anchor, gamma, beta, eps):
        y, mean, rstd = NN.layernorm_fwd(x.contiguous(), gamma.master if gamma else None,
                                         beta.master if beta else None, eps)
        ctx.gamma, ctx.beta = gamma, beta
        ctx.save_for_backward(x, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, mean, rstd = ctx.saved_tensors
        gamma, beta = ctx.gamma, ctx.beta
        acc = gamma.take_accumulate_flag() if gamma is not None else False
        if beta is not None:
            beta.take_accumulate_flag()
        dx = NN.layernorm_bwd(x.contiguous(), gamma.master if gamma else None, mean, rstd,
                              gy.contiguous().to(x.dtype), gamma.grad if gamma else None,
                              beta.grad if beta else None, acc)
        if gamma is not None:
            gamma.grad_ready()
        if beta is not None:
            beta.grad_ready()
        return dx, None, None, None, None


class DropoutFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, p, stream, seed, step_t):
        ctx.p, ctx.stream, ctx.seed, ctx.step_t = p, stream, seed, step_t
        return NN.dropout(x.contiguous(), p, stream, seed, 0, step_t)

    @staticmethod
    def backward(ctx, gy):
        return NN.dropout(gy.contiguous(), ctx.p, ctx.stream, ctx.seed, 0, ctx.step_t), None, None, None, None


class EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, table, anchor):
        ctx.table = table
        ctx.save_for_backward(ids)
        return NN.embedding_fwd(ids, table.value)

    @staticmethod
    def backward(ctx, gy):
        (ids,) = ctx.saved_tensors
        T = ctx.table
        if not T.take_accumulate_flag():
            zero_(T.grad)
        NN.embedding_bwd(ids, gy.contiguous(), T.grad)
        T.grad_ready()
        return None, None, None


class AttentionFn(torch.autograd.Function):
    """softmax(Q K^T * scale) V over a fused QKV buffer [B, S, 3*E]."""

    @staticmethod
    def forward(ctx, qkv, B, S, H, D, scale):
        out, probs = NN.attention_fwd(qkv.contiguous(), B, S, H, D, scale)
        ctx.dims = (B, S, H, D, scale)
        ctx.save_for_backward(qkv, probs, out)
        return out

    @staticmethod
    def backward(ctx, gout):
        qkv, probs, out = ctx.saved_tensors
        B, S, H, D, scale = ctx.dims
        dqkv = NN.attention_bwd(qkv, probs, gout.contiguous().to(qkv.dtype), B, S, H, D, scale, out=out)
        return dqkv, None, None, None, None, None


def softmax_cross_entropy(logits: torch.Tensor, target: torch.Tensor, reduction_scale: float):
    """Fused softmax + CE: returns (loss scalar tensor [f32], dlogits)."""
    rows_loss, dl = K.softmax_ce(logits.detach().contiguous(), target, grad_scale=reduction_scale,
                                 want_grad=True, in_place=False)
    return K.sum_scalar(rows_loss, reduction_scale), dl


class ChannelAffineFn(torch.autograd.Function):
    """y = x * gamma[c] + beta[c] over [N, C, *] (group-norm affine)."""

    @staticmethod
    def forward(ctx, x, anchor, gamma, beta):
        shape = [1, x.shape[1]] + [1] * (x.dim() - 2)
        ctx.gamma, ctx.beta, ctx.shape = gamma, beta, shape
        ctx.save_for_backward(x)
        return (x.float() * gamma.master.reshape(shape) + beta.master.reshape(shape)).to(x.dtype)

    @staticmethod
    def backward(ctx, gy):
        (x,) = ctx.saved_tensors
        gamma, beta, shape = ctx.gamma, ctx.beta, ctx.shape
        dims = [0] + list(range(2, x.dim()))
        g = gy.float()
        dg = (g * x.float()).sum(dims)
        db = g.sum(dims)
        for p, v in ((gamma, dg), (beta, db)):
            if p.take_accumulate_flag():
                p.grad.add_(v)
            else:
                p.grad.copy_(v)
            p.grad_ready()
        return (g * gamma.master.reshape(shape)).to(x.dtype), None, None, None


class TransformerBlockFn(torch.autograd.Function):
    """One pre-norm encoder block as a single autograd node:

        h1 = LN1(x);  qkv = h1 Wqkv;  a = attn(qkv);  h = a Wo + x
        h2 = LN2(h);  f = relu(h2 W1 + b1);           y = f W2 + b2 + h

    Forward fuses both residual adds and the ReLU into GEMM epilogues.  The
    hand-written backward fuses the ReLU backward into the dF GEMM epilogue
    and both residual-gradient sums into the layer-norm backward kernels, so
    a block's backward launches only this framework's kernels.
    """

    @staticmethod
    def forward(ctx, x, anchor, blk):
        B, S, E = x.shape
        H, D = blk.attn.num_heads, blk.attn.head_dim
        scale = 1.0 / math.sqrt(D)
        ln1, ln2, at, f1, f2 = blk.ln1, blk.ln2, blk.attn, blk.ff1, blk.ff2
        x2 = _flat2(x)
        h1, m1, r1 = NN.layernorm_fwd(x2, ln1.gamma.master, ln1.beta.master, ln1.eps)
        qkv = K.gemm(h1, at.w_qkv.value)
        a, probs = NN.attention_fwd(qkv.reshape(B, S, 3 * E), B, S, H, D, scale)
        a2 = _flat2(a)
        h = K.gemm(a2, at.w_o.value, residual=x2)
        h2, m2, r2 = NN.layernorm_fwd(h, ln2.gamma.master, ln2.beta.master, ln2.eps)
        # the ReLU's backward reads one bit per element instead of f
        fbits = K.relu_bits_like(h2.shape[0], f1.weight.value.shape[1], h2.device) if _RELU_BITS else None
        f = K.gemm(h2, f1.weight.value, bias=f1.bias.master, act=ACT_RELU, relu_bits_out=fbits)
        y = K.gemm(f, f2.weight.value, bias=f2.bias.master, residual=h)
        ctx.blk, ctx.dims = blk, (B, S, H, D, scale)
        ctx.save_for_backward(x2, h1, m1, r1, qkv, probs, a2, h, h2, m2, r2, f, fbits)
        return y.reshape(B, S, E)

    @staticmethod
    def backward(ctx, gy):
        x2, h1, m1, r1, qkv, probs, a2, h, h2, m2, r2, f, fbits = ctx.saved_tensors
        blk = ctx.blk
        B, S, H, D, scale = ctx.dims
        ln1, ln2, at, f1, f2 = blk.ln1, blk.ln2, blk.attn, blk.ff1, blk.ff2
        g = _flat2(gy)
        if g.dtype != x2.dtype:
            g = g.to(x2.dtype)
        g = g.contiguous()

        def wgrad(p, a_t, grad):
            K.gemm(a_t, grad, out=p.grad, beta=1.0 if p.take_accumulate_flag() else 0.0)

        def bgrad(p, grad):
            K.colsum(grad, out=p.grad, accumulate=p.take_accumulate_flag())

        # FFN: y = f W2 + b2 + h (b2's gradient, the column sums of g, comes
        # out of the LayerNorm backward below, which reads g as its residual)
        wgrad(f2.weight, f.t(), g)
        # ReLU backward and the FF1 bias gradient (column sums) fused
        mask = dict(relu_bits=fbits) if fbits is not None else dict(relu_mask=f)
        if _FUSE_COLSUM:
            df = K.gemm(g, f2.weight.value.t(), colsum_out=f1.bias.grad,
                        colsum_accumulate=f1.bias.take_accumulate_flag(), **mask)
        else:
            df = K.gemm(g, f2.weight.value.t(), **mask)
            bgrad(f1.bias, df)
        wgrad(f1.weight, h2.t(), df)
        dh2 = K.gemm(df, f1.weight.value.t())
        acc = ln2.gamma.take_accumulate_flag()
        ln2.beta.take_accumulate_flag()
        dh = NN.layernorm_bwd(h, ln2.gamma.master, m2, r2, dh2, ln2.gamma.grad, ln2.beta.grad, acc, dres=g,
                              dres_colsum=f2.bias.grad, dres_colsum_accumulate=f2.bias.take_accumulate_flag())
        # attention: h = a Wo + x
        wgrad(at.w_o, a2.t(), dh)
        da = K.gemm(dh, at.w_o.value.t())
        dqkv = NN.attention_bwd(qkv.reshape(B, S, -1), probs, da.reshape(B, S, -1), B, S, H, D, scale, out=a2)
        dqkv2 = _flat2(dqkv)
        wgrad(at.w_qkv, h1.t(), dqkv2)
        dh1 = K.gemm(dqkv2, at.w_qkv.value.t())
        acc = ln1.gamma.take_accumulate_flag()
        ln1.beta.take_accumulate_flag()
        dx = NN.layernorm_bwd(x2, ln1.gamma.master, m1, r1, dh1, ln1.gamma.grad, ln1.beta.grad, acc, dres=dh)
        # All of the block's parameter reads are enqueued: release its buckets.
        for p in (f2.weight, f2.bias, f1.weight, f1.bias, ln2.gamma, ln2.beta, at.w_o, at.w_qkv, ln1.gamma, ln1.beta):
            p.grad_ready()
        return dx.reshape(B, S, -1), None, None
