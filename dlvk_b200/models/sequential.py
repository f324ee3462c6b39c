"""`Sequential` model (include/dlvk/model/model.h:15-91,
src/model/model.cpp:20-208) with the reference's builder API.

Execution differs from the reference in three ways that keep the API:
* consecutive layers that the kernels can fuse run as one launch:
  Dense+ReLU (GEMM epilogue), Conv2D+ReLU, BatchNorm+ReLU(+Dropout);
* parameters live in flat buffers (see params.ParamStore) so the optimizer,
  checkpointing and the data-parallel all-reduce each touch one buffer;
* a trailing Softmax is fused with cross-entropy during training
  (`forward_logits` + the fused loss), which is the only configuration in
  which the reference's identity softmax-backward is correct.
"""
from __future__ import annotations

import io
import json
from typing import List, Optional

import torch

from .. import runtime
from ..ops import core as K
from . import layers as L
from .params import ParamStore

_DTYPES = {"fp32": torch.float32, "float32": torch.float32, "bf16": torch.bfloat16, "bfloat16": torch.bfloat16}


def resolve_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    return _DTYPES[str(dtype).lower()]


_CONFIG_KEYS = ("input_size", "output_size", "in_channels", "out_channels", "kernel_size", "stride", "padding",
                "pool_size", "num_features", "rate", "num_embeddings", "embedding_dim", "normalized_shape",
                "embed_dim", "num_heads", "d_model", "nhead", "dim_feedforward", "max_len", "eps", "momentum",
                "num_groups", "num_channels", "residual", "hidden_size", "num_layers", "return_sequences",
                "bidirectional", "cell", "reverse")


def layer_config(layer) -> dict:
    """Constructor arguments of one layer as a JSON-able dict."""
    d = {"type": layer.type_name}
    for k in _CONFIG_KEYS:
        v = getattr(layer, k, None)
        if isinstance(v, (int, float, bool, str)):
            d[k] = v
    if isinstance(layer, L.ActivationLayer):
        d["type"] = "Activation"
        d["activation"] = layer.activation.value
    if hasattr(layer, "bias") and hasattr(layer, "weight"):
        d["use_bias"] = layer.bias is not None
    if isinstance(layer, L.DenseLayer):
        d["activation"] = layer.activation
    if isinstance(layer, L.Conv2DLayer):
        d["activation"] = "relu" if layer.relu else None
    if isinstance(layer, L.ResidualLayer):
        d["inner"] = layer_config(layer.inner)
    return d


class Model:
    """Abstract model interface (include/dlvk/model/model.h:15-26)."""

    def forward(self, x):
        raise NotImplementedError

    def backward(self, grad_output):
        raise NotImplementedError

    def update_parameters(self, optimizer):
        raise NotImplementedError

    def set_training(self, training: bool):
        raise NotImplementedError

    def summary(self) -> str:
        raise NotImplementedError

    def parameter_count(self) -> int:
        raise NotImplementedError

    def save_weights(self, filepath: str):
        raise NotImplementedError

    def load_weights(self, filepath: str):
        raise NotImplementedError


class Sequential(Model):
    def __init__(self, device=None, dtype="fp32", seed: Optional[int] = None):
        base = device if isinstance(device, runtime.CudaDevice) else runtime.get_device(device)
        # A private RNG context: dropout masks depend on this model alone.
        self.dev = runtime.ModelContext(base, seed if seed is not None else 0)
        self.dtype = resolve_dtype(dtype)
        self.m_layers: List[L.ModernLayer] = []
        self.is_training = True
        self.store: Optional[ParamStore] = None
        self._plan = None
        self._last_out = None
        self._last_in = None
        if seed is not None:
            L.manual_seed(seed)

    # ----------------------------------------------------------- builder API
    def add(self, layer: L.ModernLayer) -> "Sequential":
        if self.store is not None:
            raise RuntimeError("cannot add layers after the model was built")
        layer.track = False
        self.m_layers.append(layer)
        self._plan = None
        return self

    add_layer = add

    def add_dense(self, input_size: int, output_size: int, use_bias: bool = True, init_std=None):
        return self.add(L.DenseLayer(input_size, output_size, use_bias, init_std=init_std))

    def add_conv2d(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1, padding: int = 0):
        return self.add(L.Conv2DLayer(in_channels, out_channels, kernel_size, stride, padding))

    def add_maxpool2d(self, pool_size: int, stride: int = 0):
        return self.add(L.MaxPool2DLayer(pool_size, stride))

    def add_avgpool2d(self, pool_size: int, stride: int = 0):
        return self.add(L.AvgPool2DLayer(pool_size, stride))

    def add_batchnorm1d(self, num_features: int):
        return self.add(L.BatchNorm1DLayer(num_features))

    def add_batchnorm2d(self, num_features: int):
        return self.add(L.BatchNorm2DLayer(num_features))

    def add_dropout(self, dropout_rate: float):
        return self.add(L.DropoutLayer(dropout_rate))

    def add_relu(self):
        return self.add(L.ActivationLayer(L.ActivationType.ReLU))

    def add_sigmoid(self):
        return self.add(L.ActivationLayer(L.ActivationType.Sigmoid))

    def add_tanh(self):
        return self.add(L.ActivationLayer(L.ActivationType.Tanh))

    def add_softmax(self):
        return self.add(L.ActivationLayer(L.ActivationType.Softmax))

    def add_flatten(self):
        return self.add(L.FlattenLayer())

    def add_embedding(self, num_embeddings: int, embedding_dim: int, init_std: float = 1.0):
        return self.add(L.EmbeddingLayer(num_embeddings, embedding_dim, init_std))

    def add_layernorm(self, normalized_shape: int, eps: float = 1e-5):
        return self.add(L.LayerNormLayer(normalized_shape, eps))

    def add_multihead_attention(self, embed_dim: int, num_heads: int, residual: bool = False, init_std=None):
        return self.add(L.MultiHeadAttentionLayer(embed_dim, num_heads, 0.0, init_std, residual))

    def add_transformer_encoder(self, d_model: int, nhead: int, dim_feedforward: int = 2048, init_std=None):
        return self.add(L.TransformerEncoderLayer(d_model, nhead, dim_feedforward, 0.0, init_std))

    def add_positional_encoding(self, d_model: int, max_len: int = 5000):
        return self.add(L.PositionalEncodingLayer(d_model, max_len))

    def add_rnn(self, input_size: int, hidden_size: int, return_sequences: bool = True):
        return self.add(L.RNNLayer(input_size, hidden_size, return_sequences))

    def add_lstm(self, input_size: int, hidden_size: int, return_sequences: bool = True):
        return self.add(L.LSTMLayer(input_size, hidden_size, return_sequences))

    def add_gru(self, input_size: int, hidden_size: int, return_sequences: bool = True):
        return self.add(L.GRULayer(input_size, hidden_size, return_sequences))

    def add_bidirectional(self, cell: str, input_size: int, hidden_size: int, return_sequences: bool = True):
        return self.add(L.BidirectionalRNN(cell, input_size, hidden_size, return_sequences))

    # ----------------------------------------------------------- build
    def build(self) -> "Sequential":
        if self.store is None:
            for layer in self.m_layers:
                layer.bind_runtime(self.dev, self.dtype)
            params = self.parameters()
            self.store = ParamStore(params, self.dev.device, self.dtype)
            self._plan = None
        return self

    def parameters(self):
        out = []
        for layer in self.m_layers:
            out.extend(layer.parameters())
        return out

    def _make_plan(self):
        """Group layers into fused execution steps."""
        plan = []
        ls = self.m_layers
        i = 0
        A = L.ActivationType
        while i < len(ls):
            cur = ls[i]
            nxt = ls[i + 1] if i + 1 < len(ls) else None
            is_relu = isinstance(nxt, L.ActivationLayer) and nxt.activation == A.ReLU
            if isinstance(cur, L.DenseLayer) and is_relu and cur._act == K.ACT_NONE:
                # Dense+ReLU feeding another Dense: the consumer's dX GEMM
                # applies this ReLU's backward in its epilogue.
                feeds_dense = i + 2 < len(ls) and isinstance(ls[i + 2], L.DenseLayer)
                mask_in = bool(plan) and getattr(plan[-1][0], "relu_feeds_dense", False)
                fn = (lambda x, c=cur, d=feeds_dense, m=mask_in:
                      c._forward(x, act=K.ACT_RELU, mask_input=m, defer_relu=d))
                fn.relu_feeds_dense = feeds_dense
                plan.append((fn, 2))
                i += 2
                continue
            if isinstance(cur, L.DenseLayer) and plan and getattr(plan[-1][0], "relu_feeds_dense", False):
                plan.append((lambda x, c=cur: c._forward(x, mask_input=True), 1))
                i += 1
                continue
            if isinstance(cur, L.Conv2DLayer) and is_relu:
                plan.append((lambda x, c=cur: c._forward(x, relu=True), 2))
                i += 2
                continue
            if isinstance(cur, L._BatchNormBase) and is_relu:
                third = ls[i + 2] if i + 2 < len(ls) else None
                if isinstance(third, L.DropoutLayer):
                    plan.append((lambda x, c=cur, d=third: c._forward(x, relu=True, p=d.rate, stream=d.stream), 3))
                    i += 3
                else:
                    plan.append((lambda x, c=cur: c._forward(x, relu=True), 2))
                    i += 2
                continue
            if isinstance(cur, L.EmbeddingLayer):
                plan.append((lambda x, c=cur: c.forward(x), 1))
            else:
                plan.append((lambda x, c=cur: c._forward(x), 1))
            i += 1
        return plan

    def _prepare_input(self, x):
        from ..tensor import Tensor as FacadeTensor

        if isinstance(x, FacadeTensor):
            x = x.data
        if x.device != self.dev.device:
            x = x.to(self.dev.device, non_blocking=True)
        if x.is_floating_point() and x.dtype != self.dtype:
            x = K.unary(x, K.UN_COPY, out_dtype=self.dtype)
        return x

    def _run(self, x, upto: Optional[int] = None):
        self.build()
        if self._plan is None:
            self._plan = self._make_plan()
        consumed = 0
        from ..utils.profiling import NVTX_LAYERS, nvtx_range

        for fn, n in self._plan:
            if upto is not None and consumed + n > upto:
                break
            if NVTX_LAYERS:
                with nvtx_range("+".join(l.type_name for l in self.m_layers[consumed:consumed + n])):
                    x = fn(x)
            else:
                x = fn(x)
            for layer in self.m_layers[consumed:consumed + n]:
                layer.output_shape = tuple(x.shape)
            consumed += n
        return x

    def has_trailing_softmax(self) -> bool:
        last = self.m_layers[-1] if self.m_layers else None
        return isinstance(last, L.ActivationLayer) and last.activation == L.ActivationType.Softmax

    # ----------------------------------------------------------- Model API
    def forward(self, x):
        from ..tensor import Tensor as FacadeTensor

        facade = isinstance(x, FacadeTensor)
        x = self._prepare_input(x)
        with torch.set_grad_enabled(self.is_training):
            y = self._run(x)
        self._last_out = y
        return FacadeTensor.wrap(y) if facade else y

    __call__ = forward

    def forward_logits(self, x):
        """Forward pass without a trailing Softmax (used with the fused CE loss)."""
        x = self._prepare_input(x)
        n = len(self.m_layers) - (1 if self.has_trailing_softmax() else 0)
        with torch.set_grad_enabled(self.is_training):
            y = self._run(x, upto=n)
        self._last_out = y
        return y

    def backward(self, grad_output):
        """Backpropagate `grad_output` (gradient w.r.t. the last forward output)."""
        from ..tensor import Tensor as FacadeTensor

        g = grad_output.data if isinstance(grad_output, FacadeTensor) else grad_output
        if self._last_out is None or not self._last_out.requires_grad:
            raise RuntimeError("backward() needs a preceding forward() in training mode")
        torch.autograd.backward(self._last_out, g.to(self._last_out.device, self._last_out.dtype))
        self.store.finish_backward()

    def zero_grad(self):
        self.build()
        self.store.zero_grad()

    def update_parameters(self, optimizer):
        optimizer.step(self)

    def set_training(self, training: bool):
        self.is_training = bool(training)
        for layer in self.m_layers:
            layer.set_training(training)

    def summary(self) -> str:
        lines = ["Model: Sequential", "-" * 60, f"{'Layer (type)':<24}{'Output Shape':<24}{'Param #':>12}", "=" * 60]
        for layer in self.m_layers:
            lines.append(layer.summary_line())
        lines.append("=" * 60)
        lines.append(f"Total params: {self.parameter_count()}")
        return "\n".join(lines)

    def parameter_count(self) -> int:
        return sum(layer.parameter_count() for layer in self.m_layers)

    def state_tensors(self):
        out = []
        for i, layer in enumerate(self.m_layers):
            for name, t in layer.state_tensors():
                out.append((f"layers.{i}.{name}", t))
        return out

    def architecture(self) -> list:
        """Per-layer constructor arguments (enough to rebuild the model with
        `models.builder.model_from_architecture`)."""
        return [layer_config(layer) for layer in self.m_layers]

    def save_weights(self, filepath: str, optimizer=None, extra_meta: Optional[dict] = None):
        from ..utils import dlvk_io

        self.build()
        dlvk_io.save_model(filepath, self, optimizer=optimizer, extra_meta=extra_meta)

    def load_weights(self, filepath: str, optimizer=None):
        from ..utils import dlvk_io

        self.build()
        dlvk_io.load_model(filepath, self, optimizer=optimizer)

    def clone(self) -> "Sequential":
        c = Sequential(self.dev, self.dtype)
        for layer in self.m_layers:
            c.add(layer.clone())
        c.is_training = self.is_training
        return c

    def size(self) -> int:
        return len(self.m_layers)

    def __len__(self):
        return len(self.m_layers)

    def __getitem__(self, i):
        return self.m_layers[i]

    def layers(self):
        return list(self.m_layers)

    # ----------------------------------------------------------- fast training step
    def train_step(self, x, y, loss_fn, optimizer, grad_hook=None):
        """One forward/backward/update.  Returns the loss as a device scalar
        (no host synchronisation)."""
        self.build()
        self.store.zero_grad()
        self.dev.advance_step()
        fused = getattr(loss_fn, "fuses_softmax", False) and self.has_trailing_softmax()
        out = self.forward_logits(x) if fused else self.forward(x)
        loss, dout = loss_fn.value_and_grad(out, y, from_logits=fused)
        torch.autograd.backward(out, dout)
        self.store.finish_backward()
        if grad_hook is not None:
            grad_hook(self)
        optimizer.step(self)
        return loss
