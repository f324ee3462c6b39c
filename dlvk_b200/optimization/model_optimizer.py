"""`ModelOptimizer` (include/dlvk/optimization/model_optimizer.h:19-265; every
body in src/optimization/model_optimizer.cpp is empty or returns constants,
and benchmark_model times an empty loop, :150-184).

Implemented here:
* quantize_model: symmetric int8 weights per output channel (the reference
  config's defaults), dynamic symmetric int8 activations per row, int32
  accumulation on the tensor cores (tcgen05 kind::i8) and an fp32
  dequantisation + bias + ReLU epilogue;
* prune_model: the reference's four PruningStrategy values
  (model_optimizer.h:30-35): magnitude (global or per layer), structured
  (whole output neurons / channels by L2 norm), gradual (cubic sparsity
  schedule, prune_step) and lottery ticket (magnitude masks, survivors
  rewound to the remembered initial weights); masks are kept so the
  sparsity survives further training steps;
* distill_model: soft-target training of a student against a teacher;
* optimize_for_inference: evaluation mode + batch-norm folding is left to the
  layers; returns the model ready for a captured graph;
* benchmark_model: device-timed latency / throughput with CUDA events, per
  batch size when `batch_sizes` is given (BenchmarkResults).
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


class PruningStrategy(enum.Enum):
    MAGNITUDE = 0
    STRUCTURED = 1
    GRADUAL = 2
    LOTTERY_TICKET = 3


@dataclass
class PruningConfig:
    """Fields of include/dlvk/optimization/model_optimizer.h:51-58.
    `sparsity` is the reference's sparsity_ratio; `structured=True` selects
    PruningStrategy.STRUCTURED.  `pruned_layers` / `skip_layers` name layers
    by index ("3" or "layers.3") or type name ("Dense"); an empty
    `pruned_layers` means every layer with a weight matrix or filter bank."""

    sparsity: float = 0.5
    structured: bool = False
    global_pruning: bool = True
    fine_tune_epochs: int = 0
    strategy: PruningStrategy = PruningStrategy.MAGNITUDE
    pruned_layers: List[str] = field(default_factory=list)
    skip_layers: List[str] = field(default_factory=list)
    gradual_pruning: bool = False
    pruning_frequency: int = 100


@dataclass
class BenchmarkResults:
    """model_optimizer.h:173-178.  average_gpu_utilization is the device-busy
    share (CUDA-event time over host wall time) of the timed loop, in
    percent; 0 on CPU.  peak_memory_usage is the caching allocator's peak
    in bytes during the runs (0 on CPU)."""

    latency_per_batch_size: dict = field(default_factory=dict)     # batch -> ms
    throughput_per_batch_size: dict = field(default_factory=dict)  # batch -> samples/s
    peak_memory_usage: int = 0
    average_gpu_utilization: float = 0.0


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


class QuantizedConv2DLayer(L.ModernLayer):
    """Inference-only int8 convolution: im2col patches quantised per row
    (dynamic, symmetric), weights per output channel, int32 accumulation in
    the int8 GEMM (tcgen05 kind::i8 when the reduction length allows, which
    the patch width is zero-padded to a multiple of 16 for) and an fp32
    dequantisation + bias + ReLU epilogue; output NCHW."""

    type_name = "QuantizedConv2D"

    def __init__(self, conv: L.Conv2DLayer, act: int = K.ACT_NONE):
        super().__init__()
        W = conv.weight.master.detach()
        self.cin, self.cout, self.k = conv.in_channels, conv.out_channels, conv.kernel_size
        self.stride, self.padding = conv.stride, conv.padding
        self.kdim = self.cin * self.k * self.k
        self.kpad = (self.kdim + 15) // 16 * 16
        w2 = torch.zeros(self.cout, self.kpad, device=W.device)
        w2[:, :self.kdim] = W.reshape(self.cout, -1).float()
        self.wq, self.w_scale = Q.quantize_rows(w2)
        self.bias = conv.bias.master.detach().clone() if conv.bias is not None else None
        self.act = act

    def parameter_count(self) -> int:
        return self.cout * self.kdim + (self.bias.numel() if self.bias is not None else 0)

    def nbytes(self) -> int:
        return self.wq.numel() + self.w_scale.numel() * 4 + (self.bias.numel() * 4 if self.bias is not None else 0)

    def _forward(self, x):
        n, _, h, w = x.shape
        ho = (h + 2 * self.padding - self.k) // self.stride + 1
        wo = (w + 2 * self.padding - self.k) // self.stride + 1
        cols = torch.nn.functional.unfold(x.float(), self.k, padding=self.padding, stride=self.stride)
        patches = cols.transpose(1, 2).reshape(n * ho * wo, self.kdim)
        if self.kpad != self.kdim:
            patches = torch.nn.functional.pad(patches, (0, self.kpad - self.kdim))
        qx, sx = Q.quantize_rows(patches.contiguous())
        y = Q.gemm_i8(qx, self.wq, sx, self.w_scale, self.bias, self.act, torch.float32)
        return y.reshape(n, ho * wo, self.cout).transpose(1, 2).reshape(n, self.cout, ho, wo).contiguous()

    def forward(self, x):
        with torch.no_grad():
            return self._forward(x)

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
            if isinstance(layer, (QuantizedDenseLayer, QuantizedConv2DLayer)):
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
        self._initial = None

    # ------------------------------------------------------------ quantisation
    def quantize_model(self, model: Optional[Sequential] = None, config: QuantizationConfig = None):
        """Returns an inference model whose Dense and Conv2D layers run in
        int8 (per-output-channel weights, dynamic per-row activations; the
        reference config's defaults, include/dlvk/optimization/
        model_optimizer.h:40-47)."""
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
            if isinstance(cur, L.Conv2DLayer):
                relu = cur.relu or (isinstance(nxt, L.ActivationLayer) and nxt.activation == A.ReLU)
                q = QuantizedConv2DLayer(cur, K.ACT_RELU if relu else K.ACT_NONE)
                steps.append(q._forward)
                i += 2 if (isinstance(nxt, L.ActivationLayer) and nxt.activation == A.ReLU) else 1
                continue
            steps.append(cur._forward)
            i += 1
        qm = _QuantizedSequential(steps, model.dev.device)
        self.stats.original_size_mb = _model_bytes(model) / 2 ** 20
        self.stats.optimized_size_mb = qm.size_bytes() / 2 ** 20
        self.stats.compression_ratio = self.stats.original_size_mb / max(self.stats.optimized_size_mb, 1e-9)
        return qm

    # ------------------------------------------------------------ pruning
    @staticmethod
    def _selected(i: int, layer, config: PruningConfig) -> bool:
        names = {str(i), f"layers.{i}", layer.type_name.lower()}
        if any(n.lower() in names for n in config.skip_layers):
            return False
        return not config.pruned_layers or any(n.lower() in names for n in config.pruned_layers)

    def _prunable(self, model: Sequential, config: PruningConfig):
        """(weight, bias) parameter pairs of the selected layers: every
        parameter with two or more dimensions, with its layer's 1-D bias
        when the layer has exactly one weight (Dense, Conv2D)."""
        out = []
        for i, layer in enumerate(model.layers()):
            if not self._selected(i, layer, config):
                continue
            ps = layer.parameters()
            ws = [p for p in ps if len(p.shape) >= 2]
            bias = getattr(layer, "bias", None) if len(ws) == 1 else None
            out.extend((w, bias if isinstance(bias, type(w)) else None) for w in ws)
        return out

    @staticmethod
    def _kth(a: torch.Tensor, frac: float) -> torch.Tensor:
        """Threshold below or at which a fraction `frac` of `a` lies."""
        k = int(frac * a.numel())
        return a.kthvalue(k).values if k > 0 else a.min() - 1

    def remember_initial_weights(self, model: Sequential) -> None:
        """Snapshot the weights a lottery-ticket pruning rewinds to (call
        right after building the model, before training)."""
        model.build()
        self._initial = {id(p): p.master.detach().clone() for p in model.parameters()}

    def prune_model(self, model: Optional[Sequential] = None, config: PruningConfig = None,
                    sparsity: Optional[float] = None) -> float:
        """Prunes the selected layers' weights to `sparsity` (default
        config.sparsity) and returns the achieved fraction of zeros over the
        pruned tensors.

        MAGNITUDE / GRADUAL: the smallest |w| are zeroed, over all selected
        tensors at once (global_pruning) or per tensor.  A one-shot call
        with GRADUAL prunes to the full target; prune_step follows the
        schedule.
        STRUCTURED: per layer, the output units (Dense columns of W [in, out],
        Conv2D filters of W [out, in, k, k]) with the smallest L2 norm are
        zeroed together with their bias; at least one unit stays.
        LOTTERY_TICKET: magnitude masks as MAGNITUDE, then every weight is
        rewound to its remembered initial value (remember_initial_weights)
        and the mask applied."""
        model = model or self.model
        config = config or PruningConfig()
        target = float(config.sparsity if sparsity is None else sparsity)
        if not 0.0 <= target < 1.0:
            raise ValueError(f"sparsity must be in [0, 1), got {target}")
        strategy = PruningStrategy.STRUCTURED if config.structured else config.strategy
        if strategy is PruningStrategy.LOTTERY_TICKET and self._initial is None:
            raise ValueError("lottery-ticket pruning needs remember_initial_weights(model) before training")
        model.build()
        pairs = self._prunable(model, config)
        if not pairs:
            return 0.0
        masks = {}
        if strategy is PruningStrategy.STRUCTURED:
            for w, b in pairs:
                wt = w.master.detach()
                unit_norm = wt.norm(dim=0) if wt.dim() == 2 else wt.reshape(wt.shape[0], -1).norm(dim=1)
                drop = min(int(target * unit_norm.numel()), unit_norm.numel() - 1)
                keep = torch.ones_like(unit_norm, dtype=torch.bool)
                if drop > 0:
                    keep[unit_norm.argsort()[:drop]] = False
                masks[id(w)] = (keep.reshape(1, -1) if wt.dim() == 2 else
                                keep.reshape(-1, *([1] * (wt.dim() - 1)))).expand_as(wt).clone()
                if b is not None:
                    masks[id(b)] = keep.clone()
        elif config.global_pruning:
            allw = torch.cat([w.master.detach().abs().reshape(-1) for w, _ in pairs])
            thr = self._kth(allw, target)
            for w, _ in pairs:
                masks[id(w)] = w.master.detach().abs() > thr
        else:
            for w, _ in pairs:
                masks[id(w)] = w.master.detach().abs() > self._kth(w.master.detach().abs().reshape(-1), target)
        by_id = {id(p): p for w, b in pairs for p in (w, b) if p is not None}
        for pid, mask in masks.items():
            p = by_id[pid]
            if strategy is PruningStrategy.LOTTERY_TICKET:
                p.master.copy_(self._initial[pid].to(p.master.device))
            p.master.mul_(mask)
            self._masks[pid] = mask
        if strategy is PruningStrategy.LOTTERY_TICKET:
            # The rest of the model (biases, norms) rewinds too.
            for p in model.parameters():
                if id(p) not in masks and id(p) in self._initial:
                    p.master.copy_(self._initial[id(p)].to(p.master.device))
        model.store.sync_value()
        zeros = sum(int((~masks[id(w)]).sum()) for w, _ in pairs)
        total = sum(w.numel for w, _ in pairs)
        self.stats.sparsity = zeros / max(total, 1)
        return self.stats.sparsity

    @staticmethod
    def gradual_sparsity(step: int, total_steps: int, final_sparsity: float) -> float:
        """Cubic schedule of Zhu and Gupta, "To prune, or not to prune"
        (2017): s_t = s_f (1 - (1 - t / T)^3), reaching s_f at t = T."""
        f = min(max(step / max(total_steps, 1), 0.0), 1.0)
        return final_sparsity * (1.0 - (1.0 - f) ** 3)

    def prune_step(self, model: Sequential, step: int, total_steps: int, config: PruningConfig = None) -> float:
        """Gradual pruning inside a training loop: every
        `config.pruning_frequency` steps the selected weights are pruned to
        the schedule's sparsity; on the other steps the masks are
        re-applied.  Returns the sparsity target in force."""
        config = config or PruningConfig(strategy=PruningStrategy.GRADUAL, gradual_pruning=True)
        target = self.gradual_sparsity(step, total_steps, config.sparsity)
        if step % max(config.pruning_frequency, 1) == 0 or step >= total_steps:
            self.prune_model(model, config, sparsity=target)
        else:
            self.apply_masks(model)
        return target

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

    @staticmethod
    def import_from_onnx(path: str, device=None) -> Sequential:
        """Rebuild a model from an ONNX file written by export_to_onnx
        (architecture from the file's metadata, weights from its
        initializers); reference include/dlvk/optimization/model_optimizer.h:149-152."""
        from ..export import ModelExportManager, ModelFormat

        model, _ = ModelExportManager().import_model(path, ModelFormat.ONNX, device)
        return model

    # ------------------------------------------------------------ benchmarking
    def benchmark_model(self, model, input_shape, iterations: int = 50, warmup: int = 5, device=None,
                        batch_sizes=None):
        """Latency and throughput of model.forward, timed with CUDA events on
        the GPU (wall clock on CPU).

        Without `batch_sizes`, `input_shape` includes the batch dimension and
        a dict {latency_ms, throughput_samples_per_s, iterations} is
        returned.  With `batch_sizes` (the reference's form,
        model_optimizer.h:166-185), `input_shape` is one sample's shape and a
        BenchmarkResults with one entry per batch size is returned."""
        dev = torch.device(device) if device else (model.dev.device if hasattr(model, "dev") else
                                                   torch.device("cuda" if torch.cuda.is_available() else "cpu"))
        if hasattr(model, "set_training"):
            model.set_training(False)
        if batch_sizes is None:
            ms, _ = self._time_forward(model, torch.rand(*input_shape, device=dev), iterations, warmup)
            return {"latency_ms": ms, "throughput_samples_per_s": input_shape[0] / (ms / 1e3),
                    "iterations": iterations}
        res = BenchmarkResults()
        if dev.type == "cuda":
            torch.cuda.reset_peak_memory_stats(dev)
        busy = wall = 0.0
        for b in batch_sizes:
            ms, wall_ms = self._time_forward(model, torch.rand(int(b), *input_shape, device=dev), iterations, warmup)
            res.latency_per_batch_size[int(b)] = ms
            res.throughput_per_batch_size[int(b)] = int(b) / (ms / 1e3)
            busy += ms * iterations
            wall += wall_ms
        if dev.type == "cuda":
            res.peak_memory_usage = int(torch.cuda.max_memory_allocated(dev))
            res.average_gpu_utilization = 100.0 * min(busy / max(wall, 1e-9), 1.0)
        return res

    @staticmethod
    def _time_forward(model, x, iterations: int, warmup: int):
        """(ms per forward, wall ms of the whole timed loop)."""
        for _ in range(warmup):
            model.forward(x)
        if x.is_cuda:
            torch.cuda.synchronize(x.device)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            s.record()
            for _ in range(iterations):
                model.forward(x)
            e.record()
            e.synchronize()
            wall = (time.perf_counter() - t0) * 1e3
            return s.elapsed_time(e) / iterations, wall
        t0 = time.perf_counter()
        for _ in range(iterations):
            model.forward(x)
        wall = (time.perf_counter() - t0) * 1e3
        return wall / iterations, wall


# ------------------------------------------------------------ architecture search
@dataclass
class SearchSpace:
    """Candidate values per gene (include/dlvk/optimization/
    model_optimizer.h:221-229)."""
    layer_widths: List[int] = field(default_factory=lambda: [32, 64, 128, 256])
    layer_depths: List[int] = field(default_factory=lambda: [1, 2, 3])
    activation_functions: List[str] = field(default_factory=lambda: ["relu", "tanh", "sigmoid"])
    dropout_rates: List[float] = field(default_factory=lambda: [0.0, 0.1, 0.3])


@dataclass
class SearchConfig:
    """Genetic-search settings (model_optimizer.h:231-238) plus the model's
    input / output sizes and a seed.  fitness_function(model) -> float,
    higher is better."""
    search_space: SearchSpace = field(default_factory=SearchSpace)
    population_size: int = 20
    num_generations: int = 50
    mutation_rate: float = 0.1
    crossover_rate: float = 0.7
    fitness_function: Optional[object] = None
    input_size: int = 784
    output_size: int = 10
    elite: int = 2
    tournament: int = 3
    seed: int = 0


class NeuralArchitectureSearch:
    """Evolutionary search over MLP architectures: a genome is a list of
    hidden layers (width, activation, dropout) whose length is one of the
    allowed depths; the phenotype is a Sequential of Dense layers with those
    activations and dropouts and a Softmax output.  Each generation keeps the
    `elite` best, then fills the population with children of tournament-
    selected parents (one-point crossover with probability crossover_rate,
    then per-gene mutation with probability mutation_rate, a depth change
    included).  The reference declares this interface with a skeleton body
    (src/optimization/model_optimizer.cpp:248-315)."""

    def __init__(self, config: SearchConfig, device=None, dtype="fp32"):
        import random

        self.cfg = config
        self.device = device
        self.dtype = dtype
        self.rng = random.Random(config.seed)
        self.history = []  # (generation, best fitness, best genome)
        self._cache = {}

    # ---- genomes
    def _gene(self):
        sp = self.cfg.search_space
        return (self.rng.choice(sp.layer_widths), self.rng.choice(sp.activation_functions),
                self.rng.choice(sp.dropout_rates))

    def generate_random_architecture(self):
        depth = self.rng.choice(self.cfg.search_space.layer_depths)
        return tuple(self._gene() for _ in range(depth))

    def mutate_architecture(self, genome):
        sp, p = self.cfg.search_space, self.cfg.mutation_rate
        out = []
        for w, a, d in genome:
            if self.rng.random() < p:
                w = self.rng.choice(sp.layer_widths)
            if self.rng.random() < p:
                a = self.rng.choice(sp.activation_functions)
            if self.rng.random() < p:
                d = self.rng.choice(sp.dropout_rates)
            out.append((w, a, d))
        if self.rng.random() < p:  # depth mutation: grow or shrink within the allowed depths
            depth = self.rng.choice(sp.layer_depths)
            while len(out) < depth:
                out.append(self._gene())
            out = out[:depth]
        return tuple(out)

    def crossover_architectures(self, g1, g2):
        depths = self.cfg.search_space.layer_depths
        cut1 = self.rng.randint(0, len(g1))
        cut2 = self.rng.randint(0, len(g2))
        child = list(g1[:cut1] + g2[cut2:])
        if len(child) not in depths:  # keep the child inside the search space
            depth = min(depths, key=lambda d: abs(d - len(child)))
            while len(child) < depth:
                child.append(self._gene())
            child = child[:depth]
        return tuple(child)

    # ---- phenotype
    def build(self, genome, seed: int = 0) -> Sequential:
        m = Sequential(self.device, self.dtype, seed=seed)
        prev = self.cfg.input_size
        for w, a, d in genome:
            m.add_dense(prev, w)
            {"relu": m.add_relu, "tanh": m.add_tanh, "sigmoid": m.add_sigmoid}[a]()
            if d > 0:
                m.add_dropout(d)
            prev = w
        m.add_dense(prev, self.cfg.output_size)
        m.add_softmax()
        return m

    def fitness(self, genome) -> float:
        if genome not in self._cache:
            fn = self.cfg.fitness_function
            if fn is None:
                raise ValueError("SearchConfig.fitness_function is required")
            self._cache[genome] = float(fn(self.build(genome)))
        return self._cache[genome]

    def _select(self, pop, fits):
        idx = [self.rng.randrange(len(pop)) for _ in range(max(1, self.cfg.tournament))]
        return pop[max(idx, key=lambda i: fits[i])]

    def search(self):
        """Returns (best genome, best fitness); history per generation."""
        c = self.cfg
        pop = [self.generate_random_architecture() for _ in range(c.population_size)]
        best, best_fit = None, -math.inf
        for gen in range(c.num_generations):
            fits = [self.fitness(g) for g in pop]
            order = sorted(range(len(pop)), key=lambda i: fits[i], reverse=True)
            if fits[order[0]] > best_fit:
                best, best_fit = pop[order[0]], fits[order[0]]
            self.history.append((gen, best_fit, best))
            nxt = [pop[i] for i in order[:max(0, min(c.elite, len(pop)))]]
            while len(nxt) < c.population_size:
                p1, p2 = self._select(pop, fits), self._select(pop, fits)
                child = self.crossover_architectures(p1, p2) if self.rng.random() < c.crossover_rate else p1
                nxt.append(self.mutate_architecture(child))
            pop = nxt
        return best, best_fit

    @staticmethod
    def search_architecture(config: SearchConfig, device=None) -> Sequential:
        """The reference's entry point: the best architecture found, built."""
        nas = NeuralArchitectureSearch(config, device)
        genome, _ = nas.search()
        return nas.build(genome)
