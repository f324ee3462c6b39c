"""Layers with the reference's public surface.

`ModernLayer` mirrors include/dlvk/layers/modern_layer.h:27-77 (forward,
backward, clone, update_parameters, set_training, get_layer_info,
save_weights/load_weights).  The legacy `Layer` names (DenseLayer,
Conv2DLayer, ...; include/dlvk/layers/*.h) are the concrete classes here, and
the adapter names of include/dlvk/layers/layer_adapters.h are aliases: both
styles run the same kernels, so no adapter (and none of its deep copies) is
needed.

Weights are initialised from a seeded generator (the reference drew from
std::random_device, e.g. src/layers/dense_layer.cpp:85-88) with the same
distributions: Xavier-normal sigma = sqrt(2 / (fan_in + fan_out)).
"""
from __future__ import annotations

import copy
import enum
import io
import math
import struct
from dataclasses import dataclass
from typing import List, Optional

import torch

from ..ops import core as K
from ..ops import functional as Fn
from ..ops import nn as NN
from .params import Parameter, ParamStore
from .. import runtime

_GEN = torch.Generator().manual_seed(0)


def manual_seed(seed: int) -> None:
    """Seed the generator used for weight initialisation."""
    _GEN.manual_seed(int(seed))


def _normal(shape, std: float) -> torch.Tensor:
    return torch.randn(*shape, generator=_GEN) * std


@dataclass
class LayerInfo:
    type: str
    output_shape_str: str = ""
    parameter_count: int = 0
    trainable: bool = False


class ActivationType(enum.Enum):
    ReLU = "relu"
    Sigmoid = "sigmoid"
    Tanh = "tanh"
    Softmax = "softmax"
    GELU = "gelu"
    Linear = "linear"


class ModernLayer:
    """Base class.  Subclasses implement `_forward(x)` with autograd-tracked
    ops and register parameters with `_param`."""

    type_name = "Layer"

    def __init__(self):
        self._params: List[Parameter] = []
        self._children: List["ModernLayer"] = []
        self.training = True
        self.track = True          # standalone use: cache input/output for backward()
        self._last_in = None
        self._last_out = None
        self.device_ctx: Optional[runtime.CudaDevice] = None
        self.compute_dtype = torch.float32
        self._store: Optional[ParamStore] = None
        self.output_shape = None

    # -- parameters -----------------------------------------------------------
    def _param(self, name: str, init: torch.Tensor, decay: bool = True) -> Parameter:
        p = Parameter(f"{self.type_name.lower()}.{name}", init.shape, init, decay)
        self._params.append(p)
        return p

    def _child(self, layer: "ModernLayer") -> "ModernLayer":
        self._children.append(layer)
        return layer

    def parameters(self) -> List[Parameter]:
        out = list(self._params)
        for c in self._children:
            out.extend(c.parameters())
        return out

    def parameter_count(self) -> int:
        return sum(p.numel for p in self.parameters())

    def bind_runtime(self, dev: runtime.CudaDevice, dtype) -> None:
        """Attach the device context (RNG step counter, dtype) recursively."""
        self.device_ctx = dev
        self.compute_dtype = dtype
        for c in self._children:
            c.bind_runtime(dev, dtype)
        self._on_bind()

    def _on_bind(self) -> None:
        pass

    def to(self, device=None, dtype=torch.float32) -> "ModernLayer":
        """Standalone placement: packs this layer's parameters into a private store."""
        dev = runtime.ModelContext(runtime.get_device(device))
        self.bind_runtime(dev, dtype)
        if self.parameters():
            self._store = ParamStore(self.parameters(), dev.device, dtype)
        return self

    def _ensure_placed(self, x: torch.Tensor) -> None:
        if self.device_ctx is None:
            self.to(x.device, x.dtype if x.is_floating_point() else torch.float32)

    # -- ModernLayer API --------------------------------------------------------
    def forward(self, x):
        from ..tensor import Tensor as FacadeTensor

        facade = isinstance(x, FacadeTensor)
        if facade:
            x = x.data
        self._ensure_placed(x)
        if self.track:
            if x.is_floating_point() and not x.requires_grad:
                x = x.detach().requires_grad_(True)
            self._last_in = x
        with torch.enable_grad() if self.track else _nullctx():
            y = self._forward(x)
        if self.track:
            self._last_out = y
        self.output_shape = tuple(y.shape)
        return FacadeTensor.wrap(y) if facade else y

    __call__ = forward

    def _forward(self, x):  # pragma: no cover - abstract
        raise NotImplementedError

    def backward(self, grad_output):
        """Gradient w.r.t. this layer's last input; parameter gradients land
        in their grad buffers (reference ModernLayer::backward)."""
        from ..tensor import Tensor as FacadeTensor

        facade = isinstance(grad_output, FacadeTensor)
        g = grad_output.data if facade else grad_output
        if self._last_out is None:
            raise RuntimeError("backward() called before forward()")
        if self._store is not None:
            self._store.zero_grad()
        if self._last_in is not None and self._last_in.requires_grad:
            (dx,) = torch.autograd.grad(self._last_out, self._last_in, g.to(self._last_out.dtype),
                                        allow_unused=True)
        else:
            torch.autograd.backward(self._last_out, g.to(self._last_out.dtype))
            dx = None
        return FacadeTensor.wrap(dx) if (facade and dx is not None) else dx

    def update_parameters(self, optimizer) -> None:
        optimizer.update_parameters(self.parameters())

    def set_training(self, training: bool) -> None:
        self.training = bool(training)
        for c in self._children:
            c.set_training(training)

    def get_layer_info(self) -> LayerInfo:
        shp = "x".join(str(s) for s in self.output_shape) if self.output_shape else "?"
        n = self.parameter_count()
        return LayerInfo(self.type_name, shp, n, n > 0)

    def clone(self) -> "ModernLayer":
        c = copy.copy(self)
        c.__dict__ = dict(self.__dict__)
        c._params = []
        mapping = {}
        for p in self._params:
            q = Parameter(p.name, p.shape, p.master.detach().cpu().clone(), p.decay)
            mapping[id(p)] = q
            c._params.append(q)
        for k, v in list(c.__dict__.items()):
            if isinstance(v, Parameter) and id(v) in mapping:
                c.__dict__[k] = mapping[id(v)]
        c._children = [ch.clone() for ch in self._children]
        for k, v in list(c.__dict__.items()):
            if isinstance(v, ModernLayer) and v in self._children:
                c.__dict__[k] = c._children[self._children.index(v)]
        for k in ("running_mean", "running_var"):
            if k in c.__dict__ and isinstance(c.__dict__[k], torch.Tensor):
                c.__dict__[k] = c.__dict__[k].detach().clone()
        c._store = None
        c.device_ctx = None
        c._last_in = c._last_out = None
        return c

    # Weight stream format: u32 count, then per tensor u32 nbytes + raw fp32.
    def state_tensors(self):
        """(name, tensor) of parameters and buffers; a child's names carry its
        index ("<j>.<name>") so two children of one type stay distinct."""
        out = [(p.name, p.master) for p in self._params]
        for j, c in enumerate(self._children):
            out.extend((f"{j}.{n}", t) for n, t in c.state_tensors())
        return out + self._buffers()

    def _buffers(self):
        return []

    def save_weights(self, f) -> None:
        ts = self.state_tensors()
        f.write(struct.pack("<I", len(ts)))
        for _, t in ts:
            b = t.detach().float().contiguous().cpu().numpy().tobytes()
            f.write(struct.pack("<Q", len(b)))
            f.write(b)

    def load_weights(self, f) -> None:
        ts = self.state_tensors()
        (n,) = struct.unpack("<I", f.read(4))
        if n != len(ts):
            raise ValueError(f"{self.type_name}: expected {len(ts)} tensors, file has {n}")
        for _, t in ts:
            (nb,) = struct.unpack("<Q", f.read(8))
            src = torch.frombuffer(bytearray(f.read(nb)), dtype=torch.float32).reshape(t.shape)
            t.copy_(src.to(t.device, t.dtype))
        self._sync_values()

    def _sync_values(self) -> None:
        stores = {id(p.store): p.store for p in self.parameters() if p.store is not None}
        for s in stores.values():
            s.sync_value()

    def is_training(self) -> bool:
        return self.training

    def update_weights(self, learning_rate: float) -> None:
        """The legacy Layer::update_weights (reference src/layers/dense_layer.cpp:68):
        one plain SGD step p -= learning_rate * grad on this layer's packed
        parameters, through the optimizer kernel on a GPU."""
        ps = [p for p in self.parameters() if p.store is not None]
        if ps:
            from ..optim import SGD

            SGD(learning_rate).update_parameters(ps)

    def _set_tensor(self, dst: torch.Tensor, src, what: str) -> None:
        """Copy `src` (a tensor or array of dst's element count) into a
        parameter master or a buffer in place, so a packed store keeps its
        views, then refresh the compute-dtype mirrors."""
        from ..tensor import Tensor as FacadeTensor

        if isinstance(src, FacadeTensor):
            src = src.data
        src = torch.as_tensor(src)
        if src.numel() != dst.numel():
            raise ValueError(f"{self.type_name}.{what}: expected {dst.numel()} elements, got {src.numel()}")
        dst.copy_(src.detach().reshape(dst.shape).to(dst.device, dst.dtype))
        self._sync_values()

    def summary_line(self) -> str:
        info = self.get_layer_info()
        return f"{info.type:<24}{info.output_shape_str:<24}{info.parameter_count:>12}"


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ============================================================== layers
class DenseLayer(ModernLayer):
    """y = x W + b, W [in, out] (src/layers/dense_layer.cpp:16-42)."""

    type_name = "Dense"

    def __init__(self, input_size: int, output_size: int, use_bias: bool = True, activation: Optional[str] = None,
                 init_std: Optional[float] = None):
        super().__init__()
        self.input_size, self.output_size = int(input_size), int(output_size)
        std = init_std if init_std is not None else math.sqrt(2.0 / (self.input_size + self.output_size))
        self.weight = self._param("weight", _normal((self.input_size, self.output_size), std))
        self.bias = self._param("bias", torch.zeros(self.output_size), decay=False) if use_bias else None
        self.activation = activation
        self._act = K.ACT_BY_NAME[activation]

    # Accessors of include/dlvk/layers/dense_layer.h:31-32 (fp32 masters;
    # W is [in, out]).  The setters copy in place.
    def get_weights(self) -> torch.Tensor:
        return self.weight.master

    def get_bias(self) -> Optional[torch.Tensor]:
        return self.bias.master if self.bias is not None else None

    def set_weights(self, w) -> None:
        self._set_tensor(self.weight.master, w, "weights")

    def set_bias(self, b) -> None:
        if self.bias is None:
            raise ValueError("Dense layer built with use_bias=False has no bias")
        self._set_tensor(self.bias.master, b, "bias")

    def _forward(self, x, act=None, residual=None, mask_input=False, defer_relu=False):
        a = self._act if act is None else act
        if x.dim() > 2 and x.shape[-1] != self.input_size:
            x = x.reshape(x.shape[0], -1)
        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        return Fn.dense(x, self.weight, self.bias, a, residual, mask_input, defer_relu)


class Conv2DLayer(ModernLayer):
    """NCHW convolution, weight [Cout, Cin, KH, KW] (src/layers/conv2d_layer.cpp)."""

    type_name = "Conv2D"

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1, padding: int = 0,
                 activation: Optional[str] = None, use_bias: bool = True):
        super().__init__()
        self.in_channels, self.out_channels = int(in_channels), int(out_channels)
        self.kernel_size, self.stride, self.padding = int(kernel_size), int(stride), int(padding)
        k2 = self.kernel_size * self.kernel_size
        std = math.sqrt(2.0 / (self.in_channels * k2 + self.out_channels * k2))
        self.weight = self._param("weight", _normal((self.out_channels, self.in_channels, self.kernel_size,
                                                     self.kernel_size), std))
        self.bias = self._param("bias", torch.zeros(self.out_channels), decay=False) if use_bias else None
        self.relu = activation == "relu"

    # Accessors of include/dlvk/layers/conv2d_layer.h:40-52; W is
    # [out_channels, in_channels, kernel, kernel].
    def get_weights(self) -> torch.Tensor:
        return self.weight.master

    def get_bias(self) -> Optional[torch.Tensor]:
        return self.bias.master if self.bias is not None else None

    def set_weights(self, w) -> None:
        self._set_tensor(self.weight.master, w, "weights")

    def set_bias(self, b) -> None:
        if self.bias is None:
            raise ValueError("Conv2D layer built with use_bias=False has no bias")
        self._set_tensor(self.bias.master, b, "bias")

    def get_in_channels(self) -> int:
        return self.in_channels

    def get_out_channels(self) -> int:
        return self.out_channels

    def get_kernel_height(self) -> int:
        return self.kernel_size

    def get_kernel_width(self) -> int:
        return self.kernel_size

    def compute_output_shape(self, input_shape) -> List[int]:
        """[N, C_out, H_out, W_out] for an [N, C_in, H, W] input (or the
        [C_in, H, W] of one image)."""
        return _window_out_shape(input_shape, self.out_channels, self.kernel_size, self.stride, self.padding)

    def _forward(self, x, relu=None):
        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        return Fn.Conv2dFn.apply(x, Fn._ANCHOR, self.weight, self.bias, self.stride, self.padding,
                                 self.relu if relu is None else relu)


def _window_out_shape(input_shape, channels: Optional[int], k: int, stride: int, pad: int) -> List[int]:
    """Output shape of a k x k window op over NCHW (or CHW) input:
    (H + 2 pad - k) // stride + 1 per spatial dimension."""
    shape = [int(d) for d in input_shape]
    if len(shape) not in (3, 4):
        raise ValueError(f"expected an NCHW or CHW shape, got {shape}")
    h, w = shape[-2:]
    ho, wo = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
    if ho <= 0 or wo <= 0:
        raise ValueError(f"window {k} with stride {stride} and padding {pad} does not fit {h}x{w}")
    return shape[:-3] + [shape[-3] if channels is None else channels, ho, wo]


class _PoolBase(ModernLayer):
    """Accessors of include/dlvk/layers/pooling_layers.h:34-38 (square
    windows, so height and width are the same)."""

    padding = 0

    def get_pool_height(self) -> int:
        return self.pool_size

    def get_pool_width(self) -> int:
        return self.pool_size

    def compute_output_shape(self, input_shape) -> List[int]:
        return _window_out_shape(input_shape, None, self.pool_size, self.stride, self.padding)


class MaxPool2DLayer(_PoolBase):
    type_name = "MaxPool2D"

    def __init__(self, pool_size: int, stride: int = 0):
        super().__init__()
        self.pool_size = int(pool_size)
        self.stride = int(stride) if stride else self.pool_size

    def _forward(self, x):
        return Fn.MaxPoolFn.apply(x, self.pool_size, self.stride)


class AvgPool2DLayer(_PoolBase):
    type_name = "AvgPool2D"

    def __init__(self, pool_size: int, stride: int = 0, padding: int = 0):
        super().__init__()
        self.pool_size = int(pool_size)
        self.stride = int(stride) if stride else self.pool_size
        self.padding = int(padding)

    def _forward(self, x):
        return Fn.AvgPoolFn.apply(x, self.pool_size, self.stride, self.padding)


class _BatchNormBase(ModernLayer):
    """Training: biased batch variance, running = (1 - m) r + m batch, m = 0.1,
    eps = 1e-5 (src/layers/batch_norm_layers.cpp:65-116); gamma = 1, beta = 0."""

    def __init__(self, num_features: int, momentum: float = 0.1, eps: float = 1e-5, affine: bool = True):
        super().__init__()
        self.num_features = int(num_features)
        self.momentum, self.eps = float(momentum), float(eps)
        self.gamma = self._param("gamma", torch.ones(self.num_features), decay=False) if affine else None
        self.beta = self._param("beta", torch.zeros(self.num_features), decay=False) if affine else None
        self.running_mean = torch.zeros(self.num_features)
        self.running_var = torch.ones(self.num_features)
        self.fuse_relu = False
        self.fuse_dropout = 0.0
        self.dropout_stream = 0

    def _on_bind(self):
        dev = self.device_ctx.device
        self.running_mean = self.running_mean.to(dev)
        self.running_var = self.running_var.to(dev)
        if not self.dropout_stream:
            self.dropout_stream = self.device_ctx.next_stream_id()

    def _buffers(self):
        return [("running_mean", self.running_mean), ("running_var", self.running_var)]

    # Accessors of include/dlvk/layers/batch_norm_layers.h:39-46; the
    # setters copy into the existing tensors (packed views stay valid).
    def get_gamma(self) -> Optional[torch.Tensor]:
        return self.gamma.master if self.gamma is not None else None

    def get_beta(self) -> Optional[torch.Tensor]:
        return self.beta.master if self.beta is not None else None

    def get_running_mean(self) -> torch.Tensor:
        return self.running_mean

    def get_running_var(self) -> torch.Tensor:
        return self.running_var

    def set_gamma(self, g) -> None:
        if self.gamma is None:
            raise ValueError("BatchNorm built with affine=False has no gamma")
        self._set_tensor(self.gamma.master, g, "gamma")

    def set_beta(self, b) -> None:
        if self.beta is None:
            raise ValueError("BatchNorm built with affine=False has no beta")
        self._set_tensor(self.beta.master, b, "beta")

    def set_running_mean(self, m) -> None:
        self._set_tensor(self.running_mean, m, "running_mean")

    def set_running_var(self, v) -> None:
        self._set_tensor(self.running_var, v, "running_var")

    def _forward(self, x, relu=False, p=0.0, stream=None):
        cfg = dict(momentum=self.momentum, eps=self.eps, training=self.training, relu=relu, p=p if self.training else 0.0,
                   stream=stream if stream is not None else self.dropout_stream, seed=self.device_ctx.seed,
                   step_t=self.device_ctx.step_t)
        return Fn.BatchNormFn.apply(x, Fn._ANCHOR, self.gamma, self.beta, self.running_mean, self.running_var, cfg)


class BatchNorm1DLayer(_BatchNormBase):
    type_name = "BatchNorm1D"


class BatchNorm2DLayer(_BatchNormBase):
    type_name = "BatchNorm2D"


class DropoutLayer(ModernLayer):
    """Inverted dropout with counter-based Philox masks (reproducible)."""

    type_name = "Dropout"

    def __init__(self, dropout_rate: float):
        super().__init__()
        self.rate = float(dropout_rate)
        self.stream = 0

    def get_dropout_rate(self) -> float:
        return self.rate

    def set_dropout_rate(self, rate: float) -> None:
        if not 0.0 <= float(rate) < 1.0:
            raise ValueError(f"dropout rate must be in [0, 1), got {rate}")
        self.rate = float(rate)

    def _on_bind(self):
        if not self.stream:
            self.stream = self.device_ctx.next_stream_id()

    def _forward(self, x):
        if not self.training or self.rate <= 0.0:
            return x
        return Fn.DropoutFn.apply(x, self.rate, self.stream, self.device_ctx.seed, self.device_ctx.step_t)


class ActivationLayer(ModernLayer):
    type_name = "Activation"

    def __init__(self, activation):
        super().__init__()
        if isinstance(activation, str):
            activation = ActivationType(activation.lower())
        self.activation = activation
        self.type_name = activation.name

    def get_activation_type(self) -> ActivationType:
        return self.activation

    def _forward(self, x):
        a = self.activation
        if a == ActivationType.Softmax:
            return Fn.SoftmaxFn.apply(x)
        if a == ActivationType.Linear:
            return x
        return Fn.ActivationFn.apply(x, a.value)


class FlattenLayer(ModernLayer):
    type_name = "Flatten"

    def _forward(self, x):
        return x.reshape(x.shape[0], -1)


class EmbeddingLayer(ModernLayer):
    """Token embedding; ids outside [0, V) produce zeros
    (shaders/embedding_lookup.comp:36-44)."""

    type_name = "Embedding"

    def __init__(self, num_embeddings: int, embedding_dim: int, init_std: float = 1.0):
        super().__init__()
        self.num_embeddings, self.embedding_dim = int(num_embeddings), int(embedding_dim)
        self.weight = self._param("weight", _normal((self.num_embeddings, self.embedding_dim), init_std))
        self._anchor = None

    def forward(self, x):
        from ..tensor import Tensor as FacadeTensor

        facade = isinstance(x, FacadeTensor)
        ids = x.data if facade else x
        if self.device_ctx is None:
            self.to(ids.device, torch.float32)
        y = Fn.EmbeddingFn.apply(ids.to(torch.int32), self.weight, Fn._ANCHOR)
        if self.track:
            self._last_in, self._last_out = None, y
        self.output_shape = tuple(y.shape)
        return FacadeTensor.wrap(y) if facade else y

    __call__ = forward

    def _forward(self, x):
        return self.forward(x)


class LayerNormLayer(ModernLayer):
    type_name = "LayerNorm"

    def __init__(self, normalized_shape: int, eps: float = 1e-5):
        super().__init__()
        self.normalized_shape, self.eps = int(normalized_shape), float(eps)
        self.gamma = self._param("gamma", torch.ones(self.normalized_shape), decay=False)
        self.beta = self._param("beta", torch.zeros(self.normalized_shape), decay=False)

    def _forward(self, x):
        return Fn.LayerNormFn.apply(x, Fn._ANCHOR, self.gamma, self.beta, self.eps)


class MultiHeadAttentionLayer(ModernLayer):
    """softmax(Q K^T / sqrt(d)) V with x W_{q,k,v,o}, W [E, E], no biases
    (src/layers/modern_layers.cpp:144-171).  Q, K and V come from one fused
    [E, 3E] projection GEMM whose output the attention kernels read in place.
    With `residual=True` the output projection adds its input (x + attn(x))
    in the GEMM epilogue."""

    type_name = "MultiHeadAttention"

    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0, init_std: Optional[float] = None,
                 residual: bool = False):
        super().__init__()
        if embed_dim % num_heads:
            raise ValueError("embed_dim must be divisible by num_heads")
        self.embed_dim, self.num_heads = int(embed_dim), int(num_heads)
        self.head_dim = self.embed_dim // self.num_heads
        std = init_std if init_std is not None else math.sqrt(2.0 / (2 * self.embed_dim))
        self.w_qkv = self._param("w_qkv", _normal((self.embed_dim, 3 * self.embed_dim), std))
        self.w_o = self._param("w_o", _normal((self.embed_dim, self.embed_dim), std))
        self.dropout = float(dropout)
        self.residual = residual

    def _forward(self, x, residual_src=None):
        B, S, E = x.shape
        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        qkv = Fn.dense(x, self.w_qkv, None)
        att = Fn.AttentionFn.apply(qkv, B, S, self.num_heads, self.head_dim, 1.0 / math.sqrt(self.head_dim))
        res = residual_src if residual_src is not None else (x if self.residual else None)
        return Fn.dense(att, self.w_o, None, K.ACT_NONE, res)


class PositionalEncodingLayer(ModernLayer):
    """Adds the sinusoidal table PE[pos, 2i] = sin(pos / 10000^(2i/d)),
    PE[pos, 2i+1] = cos(...) (src/layers/modern_layers.cpp:479-524)."""

    type_name = "PositionalEncoding"

    def __init__(self, d_model: int, max_len: int = 5000):
        super().__init__()
        self.d_model, self.max_len = int(d_model), int(max_len)
        pos = torch.arange(self.max_len, dtype=torch.float32)[:, None]
        div = torch.exp(torch.arange(0, self.d_model, 2, dtype=torch.float32) * (-math.log(10000.0) / self.d_model))
        pe = torch.zeros(self.max_len, self.d_model)
        pe[:, 0::2] = torch.sin(pos * div)
        pe[:, 1::2] = torch.cos(pos * div)[:, : pe[:, 1::2].shape[1]]
        self.table = pe
        self._cache = {}

    def _forward(self, x):
        B, S, D = x.shape
        key = (S, x.dtype, x.device)
        if key not in self._cache:
            self._cache[key] = self.table[:S].to(x.device, x.dtype).expand(B, S, D).contiguous()
        pe = self._cache[key]
        if pe.shape[0] != B:
            pe = self.table[:S].to(x.device, x.dtype).expand(B, S, D).contiguous()
            self._cache[key] = pe
        return _AddConst.apply(x, pe)


class _AddConst(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, c):
        return K.binary(x.contiguous(), c, K.BIN_ADD)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _ResidualAdd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        return K.binary(a.contiguous(), b.contiguous(), K.BIN_ADD)

    @staticmethod
    def backward(ctx, g):
        return g, g


class ResidualLayer(ModernLayer):
    """y = x + f(x) (include/dlvk/layers/modern_layers.h:217-233)."""

    type_name = "Residual"

    def __init__(self, wrapped: ModernLayer):
        super().__init__()
        self.inner = self._child(wrapped)
        self.inner.track = False

    def _forward(self, x):
        return _ResidualAdd.apply(x, self.inner._forward(x))


class GlobalAvgPoolLayer(ModernLayer):
    """[N, C, H, W] -> [N, C] mean over the spatial dims."""

    type_name = "GlobalAvgPool"

    def _forward(self, x):
        N_, C, H, W = x.shape
        return Fn.AvgPoolFn.apply(x, H, H, 0).reshape(N_, C) if H == W else x.float().mean((2, 3)).to(x.dtype)


class TransformerEncoderLayer(ModernLayer):
    """Pre-norm encoder block: x + MHA(LN(x)), then h + W2 relu(W1 LN(h))
    (include/dlvk/layers/modern_layers.h:131-160).  Both residual adds are
    fused into the output GEMMs' epilogues."""

    type_name = "TransformerEncoder"

    def __init__(self, d_model: int, nhead: int, dim_feedforward: int = 2048, dropout: float = 0.0,
                 init_std: Optional[float] = None):
        super().__init__()
        self.d_model, self.nhead, self.dim_feedforward = int(d_model), int(nhead), int(dim_feedforward)
        self.ln1 = self._child(LayerNormLayer(d_model))
        self.attn = self._child(MultiHeadAttentionLayer(d_model, nhead, dropout, init_std))
        self.ln2 = self._child(LayerNormLayer(d_model))
        self.ff1 = self._child(DenseLayer(d_model, dim_feedforward, True, "relu", init_std))
        self.ff2 = self._child(DenseLayer(dim_feedforward, d_model, True, None, init_std))
        for c in self._children:
            c.track = False

    def _forward(self, x):
        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        return Fn.TransformerBlockFn.apply(x.contiguous(), Fn._ANCHOR, self)


class GroupNormLayer(ModernLayer):
    """Group norm over [N, C, *]: layer-norm statistics per (sample, group),
    then a per-channel affine."""

    type_name = "GroupNorm"

    def __init__(self, num_groups: int, num_channels: int, eps: float = 1e-5):
        super().__init__()
        if num_channels % num_groups:
            raise ValueError("num_channels must be divisible by num_groups")
        self.num_groups, self.num_channels, self.eps = int(num_groups), int(num_channels), float(eps)
        self.gamma = self._param("gamma", torch.ones(self.num_channels), decay=False)
        self.beta = self._param("beta", torch.zeros(self.num_channels), decay=False)

    def _forward(self, x):
        N_, C = x.shape[:2]
        xr = x.reshape(N_ * self.num_groups, -1)
        y = Fn.LayerNormFn.apply(xr, Fn._ANCHOR, None, None, self.eps).reshape(x.shape)
        return Fn.ChannelAffineFn.apply(y, Fn._ANCHOR, self.gamma, self.beta)


class _RecurrentBase(ModernLayer):
    """Shared parameters and state of RNN / LSTM / GRU (weights [G*H, I] and
    [G*H, H], biases [G*H], Xavier-uniform init with bound sqrt(6/(fan_in +
    fan_out)), src/layers/recurrent_layers.cpp:70-100).  Input [B, T, I];
    output [B, T, H] (or the last step [B, H] with return_sequences=False).
    Each forward starts from the stored initial state (zeros unless set);
    the final states are kept for `get_hidden_state` / `get_cell_state`."""

    cell = "rnn"

    def __init__(self, input_size: int, hidden_size: int, return_sequences: bool = True, reverse: bool = False,
                 use_bias: bool = True):
        super().__init__()
        from ..ops.rnn import GATES, KINDS

        self.kind = KINDS[self.cell]
        self.input_size, self.hidden_size = int(input_size), int(hidden_size)
        self.return_sequences = bool(return_sequences)
        self.reverse = bool(reverse)
        G = GATES[self.kind]
        gh = G * self.hidden_size
        b_ih = math.sqrt(6.0 / (self.input_size + self.hidden_size))
        b_hh = math.sqrt(6.0 / (2 * self.hidden_size))
        self.w_ih = self._param("weight_ih", (torch.rand(gh, self.input_size) * 2 - 1) * b_ih)
        self.w_hh = self._param("weight_hh", (torch.rand(gh, self.hidden_size) * 2 - 1) * b_hh)
        if use_bias:
            bias = torch.zeros(gh)
            if self.kind == 1:
                bias[self.hidden_size:2 * self.hidden_size] = 1.0  # forget gate
            self.b_ih = self._param("bias_ih", bias, decay=False)
            self.b_hh = self._param("bias_hh", torch.zeros(gh), decay=False)
        else:
            self.b_ih = self.b_hh = None
        self.h0 = None
        self.c0 = None
        self.hidden_state = None
        self.cell_state = None

    def _directions(self):
        return [self], [self.reverse]

    def _forward(self, x):
        from ..ops.rnn import RecurrentFn

        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        cells, revs = self._directions()
        states = [(c.h0, c.c0) for c in cells]
        y = RecurrentFn.apply(x.contiguous(), Fn._ANCHOR, cells, revs, states)
        H = self.hidden_size
        last = y[:, -1] if not self.reverse else y[:, 0]
        self.hidden_state = last.detach()[..., :H]
        if self.return_sequences:
            return y
        return last

    # reference state API
    def reset_hidden_state(self):
        self.h0 = None
        self.c0 = None
        self.hidden_state = self.cell_state = None

    reset_states = reset_hidden_state

    def get_hidden_state(self):
        return self.hidden_state

    def set_hidden_state(self, h):
        self.h0 = h

    def get_cell_state(self):
        return self.cell_state

    def set_states(self, h, c):
        self.h0, self.c0 = h, c


class RNNLayer(_RecurrentBase):
    """h_t = tanh(x_t W_ih^T + b_ih + h_{t-1} W_hh^T + b_hh)."""

    type_name = "RNN"
    cell = "rnn"


class LSTMLayer(_RecurrentBase):
    """i,f,g,o = split(x W_ih^T + h W_hh^T + b); c = f c + i g; h = o tanh(c)."""

    type_name = "LSTM"
    cell = "lstm"


class GRULayer(_RecurrentBase):
    """r,z = sigma(...); n = tanh(x W_in^T + b_in + r (h W_hn^T + b_hn));
    h = (1 - z) n + z h."""

    type_name = "GRU"
    cell = "gru"


class BidirectionalRNN(ModernLayer):
    """Forward and time-reversed copies of one cell type; output [B, T, 2H]
    (both directions write their half in place)."""

    type_name = "Bidirectional"

    def __init__(self, cell_type, input_size: int, hidden_size: int, return_sequences: bool = True):
        super().__init__()
        if isinstance(cell_type, str):
            cell_type = {"rnn": RNNLayer, "lstm": LSTMLayer, "gru": GRULayer}[cell_type.lower()]
        self.cell = cell_type.cell
        self.input_size, self.hidden_size = int(input_size), int(hidden_size)
        self.return_sequences = bool(return_sequences)
        self.fwd = self._child(cell_type(input_size, hidden_size))
        self.bwd = self._child(cell_type(input_size, hidden_size, reverse=True))
        for c in self._children:
            c.track = False

    def _forward(self, x):
        from ..ops.rnn import RecurrentFn

        if x.dtype != self.compute_dtype:
            x = x.to(self.compute_dtype)
        cells = [self.fwd, self.bwd]
        y = RecurrentFn.apply(x.contiguous(), Fn._ANCHOR, cells, [False, True],
                              [(c.h0, c.c0) for c in cells])
        if self.return_sequences:
            return y
        H = self.hidden_size
        # last step of the forward direction, first step of the reverse one
        return torch.cat([y[:, -1, :H], y[:, 0, H:]], -1)


def BiLSTM(input_size: int, hidden_size: int, **kw):
    return BidirectionalRNN(LSTMLayer, input_size, hidden_size, **kw)


def BiGRU(input_size: int, hidden_size: int, **kw):
    return BidirectionalRNN(GRULayer, input_size, hidden_size, **kw)


def BiRNN(input_size: int, hidden_size: int, **kw):
    return BidirectionalRNN(RNNLayer, input_size, hidden_size, **kw)


# Reference adapter / legacy names (include/dlvk/layers/layer_adapters.h).
DenseLayerAdapter = DenseLayer
Conv2DLayerAdapter = Conv2DLayer
MaxPool2DLayerAdapter = MaxPool2DLayer
AvgPool2DLayerAdapter = AvgPool2DLayer
BatchNorm1DLayerAdapter = BatchNorm1DLayer
BatchNorm2DLayerAdapter = BatchNorm2DLayer
DropoutLayerAdapter = DropoutLayer
Layer = ModernLayer


class ConvLayer(Conv2DLayer):
    """The legacy layer of include/dlvk/layers/layer.h:22-38 (declared there,
    never defined): a stride-1, unpadded Conv2D.  The reference's trailing
    device argument is accepted and used for placement."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, device=None):
        super().__init__(in_channels, out_channels, kernel_size, 1, 0)
        if device is not None:
            self.to(getattr(device, "device", device))
