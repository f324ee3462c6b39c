"""Model optimisation: int8 quantisation, pruning, distillation, inference
preparation and benchmarking (reference include/dlvk/optimization/
model_optimizer.h)."""
from .model_optimizer import (QuantizationType, QuantizationConfig, PruningConfig, PruningStrategy, BenchmarkResults,
                              ONNXConfig, OptimizationStats,
                              ModelOptimizer, QuantizedDenseLayer)
