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
