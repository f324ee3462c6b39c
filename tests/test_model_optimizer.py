"""ModelOptimizer: int8 quantisation of Dense and Conv2D layers (against the
fp32 model) and the NeuralArchitectureSearch (seeded, deterministic, stays in
its search space, improves its fitness)."""
import pytest
import torch

from dlvk_b200.models import zoo
from dlvk_b200.optimization.model_optimizer import (ModelOptimizer, NeuralArchitectureSearch, QuantizedConv2DLayer,
                                                    QuantizedDenseLayer, SearchConfig, SearchSpace)


def _check_quantized_cnn(device):
    torch.manual_seed(0)
    m = zoo.small_cnn(device=device, dtype="fp32", seed=0)
    m.set_training(False)
    x = torch.rand(16, 1, 28, 28, device=device)
    ref = m.forward_logits(x).float()
    opt = ModelOptimizer(m)
    qm = opt.quantize_model()
    kinds = [type(getattr(fn, "__self__", None)) for fn in qm.steps]
    assert kinds.count(QuantizedConv2DLayer) == 2 and kinds.count(QuantizedDenseLayer) == 2
    y = qm.forward(x)
    probs_ref = torch.softmax(ref, -1)
    assert y.shape == probs_ref.shape
    rel = ((y.float() - probs_ref).norm() / probs_ref.norm()).item()
    assert rel < 5e-2, rel
    assert (y.argmax(-1) == probs_ref.argmax(-1)).float().mean().item() >= 0.9
    assert opt.stats.compression_ratio > 3.0


def test_int8_conv_and_dense_cpu():
    _check_quantized_cnn("cpu")


@pytest.mark.gpu
def test_int8_conv_and_dense_gpu():
    _check_quantized_cnn("cuda:0")


def _fitness(m):
    # favour ~120k parameters and ReLU layers: a known optimum inside the space
    relu = sum(1 for l in m.m_layers if str(getattr(l, "activation", "")).endswith("ReLU"))
    return -abs(m.parameter_count() - 120_000) / 1000 + relu


def test_nas_is_seeded_and_improves():
    space = SearchSpace(layer_widths=[32, 64, 128], layer_depths=[1, 2, 3], activation_functions=["relu", "tanh"],
                        dropout_rates=[0.0, 0.2])
    cfg = SearchConfig(search_space=space, population_size=12, num_generations=12, fitness_function=_fitness, seed=5)
    a = NeuralArchitectureSearch(cfg, device="cpu")
    ga, fa = a.search()
    b = NeuralArchitectureSearch(cfg, device="cpu")
    assert b.search() == (ga, fa)  # same seed, same search
    hist = [h[1] for h in a.history]
    assert all(y >= x for x, y in zip(hist, hist[1:])) and hist[-1] > hist[0]
    assert len(ga) in space.layer_depths
    for w, act, d in ga:
        assert w in space.layer_widths and act in space.activation_functions and d in space.dropout_rates
    model = NeuralArchitectureSearch.search_architecture(cfg, device="cpu")
    assert model.forward(torch.rand(4, 784)).shape == (4, 10)
