"""`ModelOptimizer` (include/dlvk/optimization/model_optimizer.h:19-265; every
body in src/optimization/model_optimizer.cpp is empty or returns constants,
and benchmark_model times an empty loop, :150-184).

Implemented here:
* quantize_model: symmetric int8 weights per output channel (the reference
  config's defaults), dynamic symmetric int8 activations per row, int32
  accumulation on the tensor cores (tcgen05 kind::i8) and an fp32
  dequantisation + bias + ReLU epilogue;
* prune_model: global or per-layer magnitude pruning (masks kept so the
  sparsity survives further training steps);
* distill_model: soft-target training of a student against a teacher;
* optimize_for_inference: evaluation mode + batch-norm folding is left to the
  layers; returns the model ready for a captured graph;
* benchmark_model: device-timed latency / throughput with CUDA events.
"""
from __future__ import annotations

import enum
import math
import time
from dataclasses import dataclass, field
from typing import List, Optional

import torch

from ..models import layers as L
from ..models.sequential import Sequential
from ..ops import core as K
from ..ops import quant as Q


class QuantizationType(enum.Enum):
    INT8 = "int8"
    FP16 = "fp16"
    BF16 = "bf16"
    DYNAMIC = "dynamic"


@dataclass
class QuantizationConfig:
    type: QuantizationType = QuantizationType.INT8
    symmetric: bool = True
    per_channel: bool = True
    calibration_samples: int = 100
    calibration_data: Optional[torch.Tensor] = None


@dataclass
class PruningConfig:
    sparsity: float = 0.5
    structured: bool = False
    global_pruning: bool = True
    fine_tune_epochs: int = 0


@dataclass
class ONNXConfig:
    opset_version: int = 13
    input_names: List[str] = field(default_factory=lambda: ["input"])
    output_names: List[str] = field(default_factory=lambda: ["output"])
    dynamic_batch: bool = True


@dataclass
class OptimizationStats:
    original_size_mb: float = 0.0
    optimized_size_mb: float = 0.0
    compression_ratio: float = 1.0
    original_latency_ms: float = 0.0
    optimized_latency_ms: float = 0.0
    speedup: float = 1.0
    accuracy_drop: float = 0.0
    sparsity: float = 0.0


class QuantizedDenseLayer(L.ModernLayer):
    """Inference-only int8 Dense: y = act(deq(q(x) @ Wq^T) + b)."""

    type_name = "QuantizedDense"

    def __init__(self, dense: L.DenseLayer, act: int = K.ACT_NONE):
        super().__init__()
        W = dense.weight.master.detach()
        wt = W.t().contiguous()                       # [out, in]: per-row == per-output-channel
        self.wq, self.w_scale = Q.quantize_rows(wt)
        self.bias = dense.bias.master.detach().clone() if dense.bias is not None else None
        self.input_size, self.output_size = dense.input_size, dense.output_size
        self.act = act
        self.out_dtype = torch.float32

    def parameter_count(self) -> int:
        return self.wq.numel() + (self.bias.numel() if self.bias is not None else 0)

    def nbytes(self) -> int:
        return self.wq.numel() + self.w_scale.numel() * 4 + (self.bias.numel() * 4 if self.bias is not None else 0)

    def _forward(self, x):
        if x.dim() > 2 and x.shape[-1] != self.input_size:
            x = x.reshape(x.shape[0], -1)
        lead = x.shape[:-1]
        qx, sx = Q.quantize_rows(x)
        y = Q.gemm_i8(qx, self.wq, sx, self.w_scale, self.bias, self.act, self.out_dtype)
        return y.reshape(*lead, self.output_size)

    def forward(self, x):
        with torch.no_grad():
            return self._forward(x if not hasattr(x, "data") or isinstance(x, torch.Tensor) else x.data)

    __call__ = forward


class _QuantizedSequential:
    """Inference-only model produced by quantize_model."""

    def __init__(self, steps, device):
        self.steps = steps
        self.device = device

    def forward(self, x):
        with torch.no_grad():
            if x.device != self.device:
                x = x.to(self.device)
            for fn in self.steps:
                x = fn(x)
            return x

    __call__ = forward

    def size_bytes(self) -> int:
        tot = 0
        for fn in self.steps:
            layer = getattr(fn, "__self__", None)
            if isinstance(layer, QuantizedDenseLayer):
                tot += layer.nbytes()
            elif isinstance(layer, L.ModernLayer):
                tot += sum(p.numel * 4 for p in layer.parameters())
        return tot


def _model_bytes(model: Sequential) -> int:
    return sum(p.numel * 4 for p in model.parameters())


class ModelOptimizer:
    def __init__(self, model: Optional[Sequential] = None):
        self.model = model
        self.stats = OptimizationStats()
        self._masks = {}

    # ------------------------------------------------------------ quantisation
    def quantize_model(self, model: Optional[Sequential] = None, config: QuantizationConfig = None):
        """Returns an inference model whose Dense layers run in int8."""
        model = model or self.model
        config = config or QuantizationConfig()
        if config.type != QuantizationType.INT8:
            raise NotImplementedError("only INT8 quantisation is implemented")
        model.build()
        model.set_training(False)
        steps = []
        ls = model.m_layers
        i = 0
        A = L.ActivationType
        while i < len(ls):
            cur = ls[i]
            nxt = ls[i + 1] if i + 1 < len(ls) else None
            if isinstance(cur, L.DenseLayer):
                relu = isinstance(nxt, L.ActivationLayer) and nxt.activation == A.ReLU
                q = QuantizedDenseLayer(cur, K.ACT_RELU if relu else K.ACT_NONE)
                steps.append(q._forward)
                i += 2 if relu else 1
                continue
            steps.append(cur._forward)
            i += 1
        qm = _QuantizedSequential(steps, model.dev.device)
        self.stats.original_size_mb = _model_bytes(model) / 2 ** 20
        self.stats.optimized_size_mb = qm.size_bytes() / 2 ** 20
        self.stats.compression_ratio = self.stats.original_size_mb / max(self.stats.optimized_size_mb, 1e-9)
        return qm

    # ------------------------------------------------------------ pruning
    def prune_model(self, model: Optional[Sequential] = None, config: PruningConfig = None) -> float:
        """Magnitude pruning of weight matrices; returns the achieved sparsity."""
        model = model or self.model
        config = config or PruningConfig()
        model.build()
        weights = [p for p in model.parameters() if len(p.shape) >= 2]
        if not weights:
            return 0.0
        if config.global_pruning:
            allw = torch.cat([p.master.detach().abs().reshape(-1) for p in weights])
            k = int(config.sparsity * allw.numel())
            thr = allw.kthvalue(max(k, 1)).values if k > 0 else allw.min() - 1
            thrs = [thr] * len(weights)
        else:
            thrs = []
            for p in weights:
                a = p.master.detach().abs().reshape(-1)
                k = int(config.sparsity * a.numel())
                thrs.append(a.kthvalue(max(k, 1)).values if k > 0 else a.min() - 1)
        zeros = 0
        total = 0
        for p, t in zip(weights, thrs):
            mask = p.master.detach().abs() > t
            p.master.mul_(mask)
            self._masks[id(p)] = mask
            zeros += int((~mask).sum())
            total += mask.numel()
        model.store.sync_value()
        self.stats.sparsity = zeros / max(total, 1)
        return self.stats.sparsity

    def apply_masks(self, model: Sequential) -> None:
        """Re-apply pruning masks (call after optimizer steps while fine-tuning)."""
        for p in model.parameters():
            m = self._masks.get(id(p))
            if m is not None:
                p.master.mul_(m)
        model.store.sync_value()

    # ------------------------------------------------------------ distillation
    def distill_model(self, teacher: Sequential, student: Sequential, x: torch.Tensor, optimizer, steps: int = 10,
                      temperature: float = 2.0) -> float:
        """Train `student` on the teacher's softened outputs (soft-target CE)."""
        from ..losses import CrossEntropyLoss

        teacher.set_training(False)
        with torch.no_grad():
            logits = teacher.forward_logits(x).float()
            soft = torch.softmax(logits / temperature, -1)
        loss = None
        for _ in range(steps):
            loss = student.train_step(x, soft, CrossEntropyLoss(), optimizer)
        return float(loss)

    # ------------------------------------------------------------ inference prep / export
    def optimize_for_inference(self, model: Optional[Sequential] = None) -> Sequential:
        model = model or self.model
        model.build()
        model.set_training(False)
        return model

    def export_to_onnx(self, model: Sequential, path: str, config: ONNXConfig = None, input_shape=None) -> bool:
        from ..export import ModelExportManager, ModelFormat

        return ModelExportManager().export_model(model, path, ModelFormat.ONNX, input_shape=input_shape)

    # ------------------------------------------------------------ benchmarking
    def benchmark_model(self, model, input_shape, iterations: int = 50, warmup: int = 5, device=None) -> dict:
        """Device-timed latency (CUDA events) and throughput of model.forward."""
        dev = torch.device(device) if device else (model.dev.device if hasattr(model, "dev") else
                                                   torch.device("cuda" if torch.cuda.is_available() else "cpu"))
        x = torch.rand(*input_shape, device=dev)
        if hasattr(model, "set_training"):
            model.set_training(False)
        for _ in range(warmup):
            model.forward(x)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iterations):
                model.forward(x)
            e.record()
            e.synchronize()
            ms = s.elapsed_time(e) / iterations
        else:
            t0 = time.perf_counter()
            for _ in range(iterations):
                model.forward(x)
            ms = (time.perf_counter() - t0) * 1e3 / iterations
        return {"latency_ms": ms, "throughput_samples_per_s": input_shape[0] / (ms / 1e3), "iterations": iterations}
