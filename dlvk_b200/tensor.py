"""`Tensor`, `TensorOps` and `TensorOpsStatic`: the reference's tensor and
op-dispatch API (include/dlvk/tensor/tensor.h:20-97,
include/dlvk/tensor/tensor_ops.h:12-199, tensor_ops_static.h:8-27) as a thin
handle over a torch tensor whose every op runs on the native kernels.

Differences that fix reference bugs: `sum(0)` returns the per-column sums
(the reference allocated shape {1} and threw, src/tensor/tensor.cpp:409-422);
tensors live in device memory, not host-visible memory; ops are
stream-ordered instead of waiting for device idle after every dispatch
(src/tensor/tensor_ops.cpp:1673-1710).
"""
from __future__ import annotations

import enum
from typing import Optional, Sequence

import numpy as np
import torch

from .ops import core as K
from .ops import nn as NN
from . import runtime


class DataType(enum.Enum):
    FLOAT32 = torch.float32
    FLOAT16 = torch.float16
    BFLOAT16 = torch.bfloat16
    INT32 = torch.int32
    INT8 = torch.int8


def _dt(d) -> torch.dtype:
    if d is None:
        return torch.float32
    if isinstance(d, DataType):
        return d.value
    return d


class Tensor:
    def __init__(self, shape: Sequence[int] = (), dtype=DataType.FLOAT32, device=None, data: Optional[torch.Tensor] = None):
        if data is not None:
            self.data = data
        else:
            dev = device.device if isinstance(device, runtime.CudaDevice) else runtime.get_device(device).device
            self.data = torch.zeros(tuple(int(s) for s in shape), dtype=_dt(dtype), device=dev)

    @staticmethod
    def wrap(t: torch.Tensor) -> "Tensor":
        return Tensor(data=t)

    @staticmethod
    def from_numpy(a, device=None) -> "Tensor":
        t = Tensor(a.shape, DataType.FLOAT32 if a.dtype == np.float32 else DataType.INT32, device)
        t.upload_data(a)
        return t

    # -- metadata -------------------------------------------------------------
    def shape(self):
        return list(self.data.shape)

    def size(self) -> int:
        return self.data.numel()

    def element_size(self) -> int:
        return self.data.element_size()

    def dtype(self):
        return self.data.dtype

    def device(self):
        return self.data.device

    # -- data transfer ----------------------------------------------------------
    def upload_data(self, src) -> None:
        if isinstance(src, torch.Tensor):
            self.data.copy_(src.reshape(self.data.shape))
        else:
            arr = np.asarray(src, dtype=np.float32 if self.data.is_floating_point() else np.int32)
            self.data.copy_(torch.from_numpy(arr.reshape(self.data.shape)).to(self.data.dtype))

    def download_data(self) -> np.ndarray:
        return self.data.detach().float().cpu().numpy() if self.data.is_floating_point() else \
            self.data.detach().cpu().numpy()

    # -- shape ops --------------------------------------------------------------
    def reshape(self, new_shape) -> "Tensor":
        return Tensor.wrap(self.data.reshape(tuple(new_shape)))

    def transpose(self, axes=None) -> "Tensor":
        if axes:
            return Tensor.wrap(self.data.permute(*axes).contiguous())
        return Tensor.wrap(K.transpose(self.data))

    # -- arithmetic ---------------------------------------------------------------
    def add(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(self.data, other.data, K.BIN_ADD))

    def add_broadcast(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.bias_act(self.data, other.data))

    def subtract(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(self.data, other.data, K.BIN_SUB))

    def multiply(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(self.data, other.data, K.BIN_MUL))

    def multiply_scalar(self, s: float) -> "Tensor":
        return Tensor.wrap(K.unary(self.data, K.UN_SCALE, float(s)))

    def divide(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(self.data, other.data, K.BIN_DIV))

    def matrix_multiply(self, other: "Tensor") -> "Tensor":
        return Tensor.wrap(K.gemm(self.data, other.data))

    def _reduce(self, op, axis: int) -> "Tensor":
        if axis == -1 or self.data.dim() == 1:
            return Tensor.wrap(K.reduce(self.data, op).reshape(1))
        if axis == 0 and self.data.dim() == 2 and op == K.RED_SUM:
            return Tensor.wrap(K.colsum(self.data))
        fn = {K.RED_SUM: torch.sum, K.RED_MAX: torch.amax, K.RED_MIN: torch.amin}[op]
        return Tensor.wrap(fn(self.data.float(), dim=axis))

    def sum(self, axis: int = -1) -> "Tensor":
        return self._reduce(K.RED_SUM, axis)

    def mean(self, axis: int = -1) -> "Tensor":
        n = self.data.numel() if (axis == -1 or self.data.dim() == 1) else self.data.shape[axis]
        s = self.sum(axis)
        return Tensor.wrap(K.unary(s.data, K.UN_SCALE, 1.0 / n))

    def max(self, axis: int = -1) -> "Tensor":
        return self._reduce(K.RED_MAX, axis)

    def min(self, axis: int = -1) -> "Tensor":
        return self._reduce(K.RED_MIN, axis)

    # -- activations ---------------------------------------------------------------
    def relu(self) -> "Tensor":
        return Tensor.wrap(K.unary(self.data, K.UN_RELU))

    def sigmoid(self) -> "Tensor":
        return Tensor.wrap(K.unary(self.data, K.UN_SIGMOID))

    def tanh(self) -> "Tensor":
        return Tensor.wrap(K.unary(self.data, K.UN_TANH))

    def softmax(self) -> "Tensor":
        return Tensor.wrap(K.softmax(self.data))

    def relu_backward(self, grad_output: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(grad_output.data, self.data, K.BIN_RELU_BWD))

    def sigmoid_backward(self, grad_output: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(grad_output.data, self.data, K.BIN_SIGMOID_BWD))

    def tanh_backward(self, grad_output: "Tensor") -> "Tensor":
        return Tensor.wrap(K.binary(grad_output.data, self.data, K.BIN_TANH_BWD))

    def __repr__(self) -> str:
        return f"dlvk.Tensor(shape={self.shape()}, dtype={self.data.dtype}, device={self.data.device})"


class TensorOps:
    """Instance op dispatcher (include/dlvk/tensor/tensor_ops.h).  Kernels are
    loaded once per process; `initialize` only checks the extension."""

    _instance: Optional["TensorOps"] = None

    def __init__(self, device=None):
        self.device = device if isinstance(device, runtime.CudaDevice) else runtime.get_device(device)

    def initialize(self) -> bool:
        return self.device.initialize()

    @classmethod
    def instance(cls) -> "TensorOps":
        if cls._instance is None:
            cls._instance = TensorOps()
        return cls._instance

    @classmethod
    def initialize_static(cls, device=None) -> bool:
        cls._instance = TensorOps(device)
        return cls._instance.initialize()

    # result-out-parameter style, returning True like the reference
    def add(self, a, b, r):
        r.data.copy_(a.add(b).data)
        return True

    def subtract(self, a, b, r):
        r.data.copy_(a.subtract(b).data)
        return True

    def multiply(self, a, b, r):
        r.data.copy_(a.multiply(b).data)
        return True

    def divide(self, a, b, r):
        r.data.copy_(a.divide(b).data)
        return True

    def matrix_multiply(self, a, b, r):
        K.gemm(a.data, b.data, out=r.data)
        return True

    def transpose(self, a, r):
        r.data.copy_(K.transpose(a.data))
        return True

    def relu(self, a, r):
        r.data.copy_(a.relu().data)
        return True

    def sigmoid(self, a, r):
        r.data.copy_(a.sigmoid().data)
        return True

    def tanh_activation(self, a, r):
        r.data.copy_(a.tanh().data)
        return True

    def softmax(self, a, r):
        r.data.copy_(a.softmax().data)
        return True

    def relu_backward(self, inp, grad, r):
        r.data.copy_(inp.relu_backward(grad).data)
        return True

    def sigmoid_backward(self, out, grad, r):
        r.data.copy_(out.sigmoid_backward(grad).data)
        return True

    def tanh_backward(self, out, grad, r):
        r.data.copy_(out.tanh_backward(grad).data)
        return True

    def copy(self, src, dst):
        dst.data.copy_(src.data)
        return True

    def fill(self, t, value: float):
        t.data.fill_(value)
        return True

    def scalar_multiply(self, a, s, r):
        r.data.copy_(a.multiply_scalar(s).data)
        return True

    def clamp(self, a, lo, hi, r):
        r.data.copy_(K.unary(a.data, K.UN_CLAMP, lo, hi))
        return True

    def sqrt(self, a, r):
        r.data.copy_(K.unary(a.data, K.UN_SQRT))
        return True

    def sum(self, a, r):
        r.data.copy_(K.reduce(a.data).reshape(r.data.shape))
        return True

    def sum_axis0(self, a, r):
        r.data.copy_(K.colsum(a.data))
        return True

    # ---- the reference's remaining instance ops (include/dlvk/tensor/
    # tensor_ops.h:28-120), each on this framework's kernels ----
    @staticmethod
    def shutdown() -> None:
        """tensor_ops.h:82: releases the singleton (kernels stay loaded)."""
        TensorOps._instance = None

    @staticmethod
    def _same_shape(*ts) -> bool:
        return all(tuple(t.shape()) == tuple(ts[0].shape()) for t in ts)

    def validate_element_wise_operation(self, a, b, r) -> bool:
        return self._same_shape(a, b, r)

    def validate_matrix_multiply(self, a, b, r) -> bool:
        sa, sb, sr = a.shape(), b.shape(), r.shape()
        return len(sa) == 2 and len(sb) == 2 and sa[1] == sb[0] and tuple(sr) == (sa[0], sb[1])

    def batch_matrix_multiply(self, a, b, r):
        """[B, M, K] x [B, K, N] -> [B, M, N] (tensor_ops.h:28), one batched
        tensor-core GEMM."""
        if a.data.dim() != 3 or b.data.dim() != 3 or a.data.shape[0] != b.data.shape[0]:
            return False
        K.gemm(a.data, b.data, out=r.data)
        return True

    def element_wise_multiply(self, a, b, r):
        return self.multiply(a, b, r)

    def element_wise_sqrt(self, a, r):
        return self.sqrt(a, r)

    def element_wise_square(self, a, r):
        r.data.copy_(K.unary(a.data, K.UN_SQUARE))
        return True

    def scale(self, a, s: float, r):
        return self.scalar_multiply(a, s, r)

    def scalar_add(self, a, s: float, r):
        r.data.copy_(K.unary(a.data, K.UN_ADD_SCALAR, s))
        return True

    def adam_update(self, gradient, m, v, param, new_m, new_v, lr: float, beta1: float, beta2: float,
                    epsilon: float) -> bool:
        """tensor_ops.h:72-74: one Adam step on `param` in place.  The
        reference's GPU path passes bias corrections of 1
        (src/tensor/tensor_ops.cpp:2330-2356), so this does too; m and v are
        updated in place and copied to new_m / new_v."""
        if not self._same_shape(gradient, m, v, param):
            return False
        from .ops.optim_kernels import make_hyper

        p = param.data
        if p.dtype != torch.float32 or not p.is_contiguous():
            return False
        if p.is_cuda:
            hyper = make_hyper(p.device, lr=lr, beta1=beta1, beta2=beta2, eps=epsilon, grad_scale=1.0,
                               bias_correction=False)
            K.N().optim_update(K.OPT_ADAM, hyper, p.view(-1), gradient.data.contiguous().view(-1), m.data.view(-1),
                               v.data.view(-1))
        else:
            g = gradient.data.float()
            m.data.mul_(beta1).add_((1 - beta1) * g)
            v.data.mul_(beta2).add_((1 - beta2) * g * g)
            p.sub_(lr * m.data / (v.data.sqrt() + epsilon))
        if new_m is not m:
            new_m.data.copy_(m.data)
        if new_v is not v:
            new_v.data.copy_(v.data)
        return True

    def gradient_clip_by_norm(self, gradient, max_norm: float, clipped) -> bool:
        """tensor_ops.h:77: clipped = g * min(1, max_norm / ||g||)."""
        g = gradient.data
        norm = float(K.reduce(g, K.RED_SUMSQ)) ** 0.5
        if norm <= max_norm:
            clipped.data.copy_(g)
        else:
            clipped.data.copy_(K.unary(g, K.UN_SCALE, max_norm / norm))
        return True

    def gradient_clip_by_value(self, gradient, min_val: float, max_val: float, clipped) -> bool:
        return self.clamp(gradient, min_val, max_val, clipped)

    def conv2d(self, inp, weights, bias, out, stride_h: int, stride_w: int, padding_h: int, padding_w: int) -> bool:
        """NCHW convolution (tensor_ops.h:86); square stride and padding."""
        if stride_h != stride_w or padding_h != padding_w:
            return False
        b = bias.data.float() if bias is not None else None
        out.data.copy_(NN.conv2d_fwd(inp.data.contiguous(), weights.data.to(inp.data.dtype), b, stride_h, padding_h))
        return True

    def conv2d_backward_input(self, grad_output, weights, grad_input, stride_h: int, stride_w: int, padding_h: int,
                              padding_w: int) -> bool:
        if stride_h != stride_w or padding_h != padding_w:
            return False
        g = grad_output.data.contiguous()
        grad_input.data.copy_(NN.conv2d_dgrad(g, weights.data.to(g.dtype), tuple(grad_input.shape()), stride_h,
                                              padding_h))
        return True

    def conv2d_backward_weight(self, inp, grad_output, grad_weights, grad_bias, stride_h: int, stride_w: int,
                               padding_h: int, padding_w: int) -> bool:
        if stride_h != stride_w or padding_h != padding_w:
            return False
        dw = torch.zeros(tuple(grad_weights.shape()), dtype=torch.float32, device=inp.data.device)
        db = torch.zeros(tuple(grad_bias.shape()), dtype=torch.float32, device=inp.data.device) \
            if grad_bias is not None else None
        NN.conv2d_wgrad(inp.data.contiguous(), grad_output.data.contiguous(), dw, db, stride_h, padding_h)
        grad_weights.data.copy_(dw)
        if db is not None:
            grad_bias.data.copy_(db)
        return True

    def maxpool2d(self, inp, out, indices, pool_h: int, pool_w: int, stride_h: int, stride_w: int,
                  padding_h: int = 0, padding_w: int = 0) -> bool:
        if pool_h != pool_w or stride_h != stride_w or padding_h or padding_w:
            return False
        y, idx = NN.maxpool_fwd(inp.data.contiguous(), pool_h, stride_h)
        out.data.copy_(y)
        indices.data.copy_(idx.to(indices.data.dtype))
        self._pool_geom = (inp.shape()[2], inp.shape()[3], pool_h, stride_h)
        return True

    def maxpool2d_backward(self, grad_output, indices, grad_input) -> bool:
        sh = grad_input.shape()
        go = grad_output.shape()
        k = getattr(self, "_pool_geom", (sh[2], sh[3], sh[2] // max(go[2], 1), sh[2] // max(go[2], 1)))
        H, W, kk, st = sh[2], sh[3], k[2], k[3]
        grad_input.data.copy_(NN.maxpool_bwd(grad_output.data.contiguous(), indices.data.to(torch.int32).contiguous(),
                                             H, W, kk, st))
        return True

    def avgpool2d(self, inp, out, pool_h: int, pool_w: int, stride_h: int, stride_w: int, padding_h: int = 0,
                  padding_w: int = 0) -> bool:
        if pool_h != pool_w or stride_h != stride_w or padding_h != padding_w:
            return False
        out.data.copy_(NN.avgpool_fwd(inp.data.contiguous(), pool_h, stride_h, padding_h))
        return True

    def avgpool2d_backward(self, grad_output, grad_input, pool_h: int, pool_w: int, stride_h: int, stride_w: int,
                           padding_h: int = 0, padding_w: int = 0) -> bool:
        if pool_h != pool_w or stride_h != stride_w or padding_h != padding_w:
            return False
        sh = grad_input.shape()
        grad_input.data.copy_(NN.avgpool_bwd(grad_output.data.contiguous(), sh[2], sh[3], pool_h, stride_h, padding_h))
        return True

    def batch_norm(self, inp, gamma, beta, running_mean, running_var, out, saved_mean, saved_var, momentum: float,
                   epsilon: float, training: bool) -> bool:
        """tensor_ops.h:107-110; saved_var receives the batch variance."""
        y, mean, rstd = NN.batchnorm_fwd(inp.data.contiguous(), gamma.data.float(), beta.data.float(),
                                         running_mean.data, running_var.data, momentum, epsilon, training)
        out.data.copy_(y)
        saved_mean.data.copy_(mean)
        saved_var.data.copy_(1.0 / (rstd.float() ** 2) - epsilon)
        return True

    def batch_norm_backward(self, grad_output, inp, gamma, saved_mean, saved_var, grad_input, grad_gamma, grad_beta,
                            epsilon: float) -> bool:
        rstd = torch.rsqrt(saved_var.data.float() + epsilon)
        dg = torch.zeros_like(gamma.data, dtype=torch.float32)
        dbb = torch.zeros_like(gamma.data, dtype=torch.float32)
        dx = NN.batchnorm_bwd(inp.data.contiguous(), grad_output.data.contiguous(), saved_mean.data.float(), rstd,
                              gamma.data.float(), None, dg, dbb, False)
        grad_input.data.copy_(dx)
        grad_gamma.data.copy_(dg)
        grad_beta.data.copy_(dbb)
        return True

    def dropout(self, inp, out, mask, dropout_rate: float, training: bool, seed: int) -> bool:
        """tensor_ops.h:117: out = inp * mask / (1 - p), mask in {0, 1}.  The
        keep pattern comes from this framework's Philox stream for `seed`, not
        the reference's xorshift hash."""
        x = inp.data
        if not training or dropout_rate <= 0:
            out.data.copy_(x)
            mask.data.fill_(1)
            return True
        keep = NN.philox_keep_mask(x.numel(), dropout_rate, int(seed), 0, 0).reshape(x.shape).to(x.device)
        mask.data.copy_(keep.to(mask.data.dtype))
        out.data.copy_(torch.where(keep, x.float() / (1 - dropout_rate), torch.zeros((), device=x.device)))
        return True

    def dropout_backward(self, grad_output, mask, grad_input, dropout_rate: float) -> bool:
        g = grad_output.data.float()
        grad_input.data.copy_(torch.where(mask.data != 0, g / (1 - dropout_rate), torch.zeros((), device=g.device)))
        return True

    def embedding_lookup(self, out, indices, embeddings) -> bool:
        out.data.copy_(NN.embedding_fwd(indices.data.to(torch.int32).contiguous(), embeddings.data))
        return True

    def layer_norm(self, out, inp, weight, bias, eps: float = 1e-5) -> bool:
        y, _, _ = NN.layernorm_fwd(inp.data.contiguous(), weight.data.float(), bias.data.float(), eps)
        out.data.copy_(y)
        return True

    def attention(self, out, query, key, value, scale: float = 1.0) -> bool:
        """out = softmax(q k^T * scale) v over the last two dims
        (tensor_ops.h:56): two tensor-core GEMMs and the row softmax."""
        q, k, v = query.data, key.data, value.data
        s = K.gemm(q, k.transpose(-1, -2), alpha=scale, out_dtype=torch.float32)
        p = K.softmax(s).to(v.dtype)
        out.data.copy_(K.gemm(p, v))
        return True

    def reshape_for_attention(self, out, inp, batch_size: int, seq_len: int, num_heads: int, head_dim: int) -> bool:
        """[B, S, H*D] -> [B, H, S, D] (tensor_ops.h:59)."""
        x = inp.data.reshape(batch_size, seq_len, num_heads, head_dim)
        out.data.copy_(K.permute4(x.contiguous(), [0, 2, 1, 3]).reshape(out.data.shape))
        return True

    def reshape_from_attention(self, out, inp, batch_size: int, seq_len: int, num_heads: int, head_dim: int) -> bool:
        """[B, H, S, D] -> [B, S, H*D] (tensor_ops.h:61)."""
        x = inp.data.reshape(batch_size, num_heads, seq_len, head_dim)
        out.data.copy_(K.permute4(x.contiguous(), [0, 2, 1, 3]).reshape(out.data.shape))
        return True


class TensorOpsStatic:
    """Static facade over TensorOps.instance() (src/tensor/tensor_ops_static.cpp:6-54)."""

    @staticmethod
    def relu(inp, result):
        return TensorOps.instance().relu(inp, result)

    @staticmethod
    def sigmoid(inp, result):
        return TensorOps.instance().sigmoid(inp, result)

    @staticmethod
    def tanh_activation(inp, result):
        return TensorOps.instance().tanh_activation(inp, result)

    @staticmethod
    def softmax(inp, result):
        return TensorOps.instance().softmax(inp, result)

    @staticmethod
    def matrix_multiply(a, b, result):
        return TensorOps.instance().matrix_multiply(a, b, result)

    @staticmethod
    def relu_backward(inp, grad_output, grad_input):
        return TensorOps.instance().relu_backward(inp, grad_output, grad_input)

    @staticmethod
    def sigmoid_backward(out, grad_output, grad_input):
        return TensorOps.instance().sigmoid_backward(out, grad_output, grad_input)

    @staticmethod
    def tanh_backward(out, grad_output, grad_input):
        return TensorOps.instance().tanh_backward(out, grad_output, grad_input)

    @staticmethod
    def copy(src, dst):
        return TensorOps.instance().copy(src, dst)

    @staticmethod
    def fill(t, value):
        return TensorOps.instance().fill(t, value)
