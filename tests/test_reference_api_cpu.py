"""CPU tests of the reference's public accessor and helper spellings: layer
get_/set_ accessors and output shapes, optimizer clipping setters,
update_parameter and zero_gradients, ModelSerializer's static entry points,
the persistence factory functions, ONNX import, LossOpsGPU, the four
pruning strategies and the per-batch-size benchmark.  Each result is checked
against plain PyTorch math or a round trip."""
import pytest
import torch
import torch.nn.functional as F

import dlvk_b200 as dl
from dlvk_b200.models import layers as L
from dlvk_b200.optimization.model_optimizer import ModelOptimizer
from dlvk_b200.training import SerializationFormat, persistence_factory
from dlvk_b200.training.persistence import ModelCheckpointCallback, ModelSerializer, ModelVersioning


def _mlp(seed):
    m = dl.Sequential("cpu", seed=seed)
    m.add_dense(6, 5)
    m.add_relu()
    m.add_dense(5, 3)
    m.add_softmax()
    return m.build()


def test_dense_get_set_weights_feed_the_forward():
    m = _mlp(0)
    d = m[0]
    assert d.get_weights().shape == (6, 5) and d.get_bias().shape == (5,)
    w = torch.randn(6, 5)
    b = torch.randn(5)
    d.set_weights(w)
    d.set_bias(b)
    assert torch.equal(d.get_weights(), w) and torch.equal(d.get_bias(), b)
    # the packed store sees the new values (set_* copies in place)
    assert torch.equal(m.store.master[d.weight.offset:d.weight.offset + 30].reshape(6, 5), w)
    x = torch.randn(4, 6)
    h = torch.relu(x @ w + b)
    ref = torch.softmax(h @ m[2].get_weights() + m[2].get_bias(), -1)
    torch.testing.assert_close(m.forward(x), ref, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        d.set_weights(torch.zeros(7))
    nb = L.DenseLayer(3, 2, use_bias=False)
    assert nb.get_bias() is None
    with pytest.raises(ValueError):
        nb.set_bias(torch.zeros(2))


@pytest.mark.parametrize("k,s,p,hw", [(3, 1, 1, 8), (3, 2, 0, 9), (5, 2, 2, 11)])
def test_conv_and_pool_output_shapes_match_forward(k, s, p, hw):
    conv = L.Conv2DLayer(2, 4, k, s, p)
    x = torch.randn(3, 2, hw, hw)
    assert conv.compute_output_shape(list(x.shape)) == list(conv.forward(x).shape)
    assert conv.compute_output_shape([2, hw, hw]) == list(conv.forward(x).shape)[1:]
    assert (conv.get_in_channels(), conv.get_out_channels()) == (2, 4)
    assert conv.get_kernel_height() == conv.get_kernel_width() == k
    assert conv.get_weights().shape == (4, 2, k, k)
    w, b = torch.randn(4, 2, k, k), torch.randn(4)
    conv.set_weights(w)
    conv.set_bias(b)
    torch.testing.assert_close(conv.forward(x), F.conv2d(x, w, b, s, p), rtol=1e-5, atol=1e-5)
    for pool in (L.MaxPool2DLayer(2, 2), L.AvgPool2DLayer(3, 2, 1)):
        assert pool.compute_output_shape(list(x.shape)) == list(pool.forward(x).shape)
        assert pool.get_pool_height() == pool.get_pool_width() == pool.pool_size
    with pytest.raises(ValueError):
        L.MaxPool2DLayer(4, 4).compute_output_shape([1, 1, 2, 2])


def test_batchnorm_accessors_drive_eval_forward():
    bn = L.BatchNorm1DLayer(4)
    g, b = torch.rand(4) + 0.5, torch.randn(4)
    rm, rv = torch.randn(4), torch.rand(4) + 0.1
    bn.set_gamma(g)
    bn.set_beta(b)
    bn.set_running_mean(rm)
    bn.set_running_var(rv)
    for get, want in ((bn.get_gamma, g), (bn.get_beta, b), (bn.get_running_mean, rm), (bn.get_running_var, rv)):
        assert torch.equal(get(), want)
    bn.set_training(False)
    assert not bn.is_training()
    x = torch.randn(8, 4)
    torch.testing.assert_close(bn.forward(x), (x - rm) / torch.sqrt(rv + bn.eps) * g + b, rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        L.BatchNorm1DLayer(4, affine=False).set_gamma(g)


def test_dropout_and_activation_accessors():
    d = L.DropoutLayer(0.25)
    assert d.get_dropout_rate() == 0.25
    d.set_dropout_rate(0.5)
    assert d.get_dropout_rate() == 0.5
    with pytest.raises(ValueError):
        d.set_dropout_rate(1.0)
    d.set_dropout_rate(0.0)
    x = torch.randn(64)
    assert torch.equal(d.forward(x), x)
    assert L.ActivationLayer("tanh").get_activation_type() == L.ActivationType.Tanh


def _sgd_ref(p, grads, lr, mu):
    p, v = p.clone(), torch.zeros_like(p)
    for g in grads:
        v = mu * v + g
        p = p - lr * v
    return p


def test_update_parameter_keeps_per_tensor_state():
    torch.manual_seed(0)
    p0 = torch.randn(10)
    grads = [torch.randn(10) for _ in range(3)]
    p = p0.clone()
    opt = dl.SGD(0.1, 0.9)
    for g in grads:
        g_before = g.clone()
        opt.update_parameter(p, g)
        assert torch.equal(g, g_before)  # the caller's gradient is not clipped or scaled in place
    torch.testing.assert_close(p, _sgd_ref(p0, grads, 0.1, 0.9), rtol=1e-6, atol=1e-7)

    # Adam with bias correction against torch.optim.Adam
    q = torch.nn.Parameter(p0.clone())
    ref = torch.optim.Adam([q], lr=1e-2, betas=(0.9, 0.999), eps=1e-8)
    mine = p0.clone()
    adam = dl.Adam(1e-2)
    for g in grads:
        q.grad = g.clone()
        ref.step()
        adam.update_parameter(mine, g)
    torch.testing.assert_close(mine, q.detach(), rtol=1e-5, atol=1e-6)


def test_update_parameter_bf16_tensor_keeps_fp32_master():
    p0 = torch.randn(32)
    p = p0.bfloat16()
    opt = dl.SGD(1e-3)
    g = torch.full((32,), 1.0)
    for _ in range(4):
        opt.update_parameter(p, g)
    # four steps of 1e-3 accumulate in the fp32 master before rounding
    torch.testing.assert_close(p.float(), (p0.bfloat16().float() - 4e-3).bfloat16().float(), rtol=0, atol=0)


def test_gradient_clipping_setters():
    g = torch.tensor([-3.0, -0.5, 0.25, 2.0])
    p = torch.zeros(4)
    opt = dl.SGD(1.0)
    opt.set_grad_clip_value(-1.0, 0.5)
    opt.update_parameter(p, g)
    torch.testing.assert_close(p, -g.clamp(-1.0, 0.5))
    with pytest.raises(ValueError):
        opt.set_grad_clip_value(1.0, -1.0)
    opt.disable_grad_clipping()
    opt.set_grad_clip_norm(1.0)
    p = torch.zeros(4)
    opt.update_parameter(p, g)
    torch.testing.assert_close(p.norm(), torch.tensor(1.0), rtol=1e-4, atol=1e-5)
    opt.disable_grad_clipping()
    p = torch.zeros(4)
    opt.update_parameter(p, g)
    torch.testing.assert_close(p, -g)
    opt.set_lr(0.5)
    assert opt.get_lr() == 0.5 == opt.get_learning_rate()


def test_zero_gradients_clears_the_store():
    m = _mlp(1)
    opt = dl.SGD(0.1)
    m.train_step(torch.randn(4, 6), torch.tensor([0, 1, 2, 0], dtype=torch.int32), dl.CrossEntropyLoss(), opt)
    assert m.store.grad.abs().sum() > 0
    opt.zero_gradients()
    assert m.store.grad.abs().sum() == 0


@pytest.mark.parametrize("fmt", [SerializationFormat.DLVK_BINARY, SerializationFormat.DLVK_JSON,
                                 SerializationFormat.NUMPY_NPZ])
def test_serializer_save_and_load_weights(tmp_path, fmt):
    src, dst = _mlp(2), _mlp(3)
    assert not torch.equal(src.store.master, dst.store.master)
    path = str(tmp_path / "w.bin")
    assert ModelSerializer.save_weights(src, path, fmt)
    assert ModelSerializer.load_weights(dst, path, fmt)
    assert torch.equal(src.store.master, dst.store.master)
    x = torch.randn(3, 6)
    assert torch.equal(src.forward(x), dst.forward(x))


def test_serializer_save_and_load_model(tmp_path):
    src = _mlp(4)
    x = torch.randn(3, 6)
    for fmt, name in ((SerializationFormat.DLVK_BINARY, "m.dlvk"), (SerializationFormat.DLVK_JSON, "m.json")):
        path = str(tmp_path / name)
        assert ModelSerializer.save_model(src, path, fmt)
        back = ModelSerializer.load_model(path, fmt, device="cpu")
        assert torch.equal(back.forward(x), src.forward(x))


def test_export_to_numpy_and_onnx_round_trip(tmp_path):
    import numpy as np

    m = _mlp(5)
    npz = str(tmp_path / "w.npz")
    assert ModelSerializer.export_to_numpy(m, npz)
    with np.load(npz) as z:
        names = [n for n, _ in m.state_tensors()]
        assert sorted(z.files) == sorted(names)
        for n, t in m.state_tensors():
            assert np.array_equal(z[n], t.numpy())
    onnx = str(tmp_path / "m.onnx")
    assert ModelSerializer.export_to_onnx(m, onnx, [[1, 6]])
    back = ModelOptimizer.import_from_onnx(onnx, device="cpu")
    x = torch.randn(2, 6)
    torch.testing.assert_close(back.forward(x), m.forward(x), rtol=0, atol=0)


def test_persistence_factory(tmp_path):
    m = _mlp(6)
    cb = persistence_factory.create_checkpoint_callback(m, str(tmp_path / "ck"), "net")
    assert isinstance(cb, ModelCheckpointCallback)
    assert cb.get_checkpoint_manager().model_name == "net"
    vs = persistence_factory.create_versioning_system(str(tmp_path / "exp"))
    assert isinstance(vs, ModelVersioning)


def test_loss_ops_gpu_entry_points_match_torch():
    torch.manual_seed(1)
    ops = dl.LossOpsGPU()
    assert ops.initialize()
    p = torch.rand(8, 5) * 0.98 + 0.01
    t = torch.rand(8, 5)
    torch.testing.assert_close(ops.mse_forward(p, t), F.mse_loss(p, t), rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(ops.mse_backward(p, t), 2 * (p - t) / p.numel(), rtol=1e-5, atol=1e-7)
    probs = torch.softmax(torch.randn(8, 5), -1)
    onehot = F.one_hot(torch.randint(0, 5, (8,)), 5).float()
    torch.testing.assert_close(ops.cross_entropy_forward(probs, onehot),
                               -(onehot * torch.log(probs + 1e-8)).sum() / 8, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(ops.cross_entropy_backward(probs, onehot), -onehot / (probs + 1e-8) / 8,
                               rtol=1e-5, atol=1e-7)
    tb = (torch.rand(8, 5) > 0.5).float()
    pe = torch.tensor([[0.0, 1e-4, 0.5, 1.0 - 1e-4, 1.0]])
    te = torch.tensor([[0.0, 1.0, 1.0, 0.0, 1.0]])
    for pp, tt in ((p, tb), (pe, te)):
        for eps in (1e-7, 1e-3):
            pc = pp.clamp(eps, 1 - eps)
            torch.testing.assert_close(ops.binary_cross_entropy_forward(pp, tt, eps),
                                       F.binary_cross_entropy(pc, tt), rtol=1e-4, atol=1e-6)
            torch.testing.assert_close(ops.binary_cross_entropy_backward(pp, tt, eps),
                                       (pc - tt) / (pc * (1 - pc)) / pp.numel(), rtol=1e-4, atol=1e-6)
    with pytest.raises(ValueError):
        ops.binary_cross_entropy_forward(p, tb, 1e-9)


# ---------------------------------------------------------------- pruning strategies
from dlvk_b200.optimization import BenchmarkResults, PruningConfig, PruningStrategy  # noqa: E402


def _prune_net(seed=0):
    m = dl.Sequential("cpu", seed=seed)
    m.add_conv2d(1, 8, 3, 1, 1)
    m.add_relu()
    m.add_flatten()
    m.add_dense(8 * 6 * 6, 16)
    m.add_relu()
    m.add_dense(16, 4)
    return m.build()


def test_magnitude_pruning_global_and_per_layer():
    for global_pruning in (True, False):
        m = _prune_net()
        ws = [p.master.clone() for p in m.parameters() if len(p.shape) >= 2]
        opt = ModelOptimizer()
        got = opt.prune_model(m, PruningConfig(sparsity=0.5, global_pruning=global_pruning))
        pruned = [p.master for p in m.parameters() if len(p.shape) >= 2]
        total = sum(w.numel() for w in ws)
        zeros = sum(int((w == 0).sum()) for w in pruned)
        assert got == pytest.approx(zeros / total)
        assert 0.49 <= got <= 0.51
        if global_pruning:
            thr = torch.cat([w.abs().reshape(-1) for w in ws]).kthvalue(int(0.5 * total)).values
            for w0, w in zip(ws, pruned):
                assert torch.equal(w, w0 * (w0.abs() > thr))
        else:
            for w0, w in zip(ws, pruned):
                assert 0.45 <= float((w == 0).float().mean()) <= 0.55
        # masks hold across a training step
        m.train_step(torch.randn(4, 1, 6, 6), torch.tensor([0, 1, 2, 3], dtype=torch.int32),
                     dl.CrossEntropyLoss(), dl.SGD(0.1))
        opt.apply_masks(m)
        assert sum(int((p.master == 0).sum()) for p in m.parameters() if len(p.shape) >= 2) >= zeros


def test_structured_pruning_zeroes_whole_units():
    m = _prune_net(1)
    conv, d1 = m[0], m[3]
    cn = conv.get_weights().reshape(8, -1).norm(dim=1)
    dn = d1.get_weights().norm(dim=0)
    conv.set_bias(torch.ones(8))
    d1.set_bias(torch.ones(16))
    ModelOptimizer().prune_model(m, PruningConfig(sparsity=0.5, strategy=PruningStrategy.STRUCTURED,
                                                   pruned_layers=["0", "Dense"], skip_layers=["layers.5"]))
    dead_c = conv.get_weights().reshape(8, -1).abs().sum(1) == 0
    assert torch.equal(dead_c, torch.isin(torch.arange(8), cn.argsort()[:4]))
    assert torch.equal(conv.get_bias() == 0, dead_c)
    dead_d = d1.get_weights().abs().sum(0) == 0
    assert torch.equal(dead_d, torch.isin(torch.arange(16), dn.argsort()[:8]))
    assert torch.equal(d1.get_bias() == 0, dead_d)
    assert int((m[5].get_weights() == 0).sum()) == 0  # skipped layer untouched


def test_gradual_schedule_and_prune_step():
    assert ModelOptimizer.gradual_sparsity(0, 100, 0.8) == 0.0
    assert ModelOptimizer.gradual_sparsity(100, 100, 0.8) == pytest.approx(0.8)
    assert ModelOptimizer.gradual_sparsity(50, 100, 0.8) == pytest.approx(0.8 * (1 - 0.5 ** 3))
    m = _prune_net(2)
    opt = ModelOptimizer()
    cfg = PruningConfig(sparsity=0.6, strategy=PruningStrategy.GRADUAL, gradual_pruning=True, pruning_frequency=5)
    last = -1.0
    for step in range(0, 21):
        opt.prune_step(m, step, 20, cfg)
        s = opt.stats.sparsity
        assert s >= last - 1e-9
        last = s
    assert last == pytest.approx(0.6, abs=0.01)


def test_lottery_ticket_rewinds_survivors():
    m = _prune_net(3)
    opt = ModelOptimizer()
    with pytest.raises(ValueError):
        opt.prune_model(m, PruningConfig(strategy=PruningStrategy.LOTTERY_TICKET))
    opt.remember_initial_weights(m)
    init = {id(p): p.master.clone() for p in m.parameters()}
    sgd = dl.SGD(0.5)
    for _ in range(3):
        m.train_step(torch.randn(8, 1, 6, 6), torch.randint(0, 4, (8,), dtype=torch.int32),
                     dl.CrossEntropyLoss(), sgd)
    trained = {id(p): p.master.clone() for p in m.parameters()}
    opt.prune_model(m, PruningConfig(sparsity=0.5, strategy=PruningStrategy.LOTTERY_TICKET))
    for p in m.parameters():
        if len(p.shape) >= 2:
            keep = trained[id(p)].abs() > 0
            alive = p.master != 0
            assert torch.equal(p.master[alive], init[id(p)][alive])
            assert int(alive.sum()) <= int(keep.sum())
        else:
            assert torch.equal(p.master, init[id(p)])


def test_benchmark_model_per_batch_size():
    m = _mlp(7)
    r = ModelOptimizer().benchmark_model(m, [6], iterations=3, warmup=1, device="cpu", batch_sizes=[1, 4])
    assert isinstance(r, BenchmarkResults)
    assert sorted(r.latency_per_batch_size) == [1, 4]
    for b, ms in r.latency_per_batch_size.items():
        assert ms > 0 and r.throughput_per_batch_size[b] == pytest.approx(b / (ms / 1e3))
    d = ModelOptimizer().benchmark_model(m, [4, 6], iterations=2, warmup=1, device="cpu")
    assert d["latency_ms"] > 0


def test_legacy_names():
    from dlvk_b200.data.transforms import PreprocessingPipeline, SimpleBuilder
    from dlvk_b200.deployment.inference import Config

    conv = dl.ConvLayer(2, 3, 3)
    x = torch.randn(1, 2, 5, 5)
    assert list(conv.forward(x).shape) == [1, 3, 3, 3]
    torch.testing.assert_close(conv.forward(x), F.conv2d(x, conv.get_weights(), conv.get_bias()),
                               rtol=1e-5, atol=1e-5)
    p = SimpleBuilder().resize(8, 8).random_horizontal_flip(0.5).normalize([0.5], [0.5]).build()
    assert isinstance(p, PreprocessingPipeline)
    assert tuple(p.process(torch.rand(2, 1, 4, 4)).shape) == (2, 1, 8, 8)
    assert Config.Serving().timeout_ms == Config().serving.timeout_ms == 1000


def test_device_getters_on_cpu():
    from dlvk_b200.runtime import CudaDevice

    d = CudaDevice("cpu")
    assert d.get_device_name() == d.get_device_type_string() == "cpu"
    assert d.get_total_device_memory() == d.get_max_memory_allocation() == 0
    assert d.get_memory_heap_count() == 0 and d.get_max_workgroup_size() == 0


def test_legacy_update_weights_is_plain_sgd():
    m = _mlp(8)
    m.train_step(torch.randn(4, 6), torch.tensor([0, 1, 2, 0], dtype=torch.int32), dl.CrossEntropyLoss(),
                 dl.SGD(0.0))
    d = m[0]
    w0, g = d.get_weights().clone(), d.weight.grad.clone()
    other = m[2].get_weights().clone()
    d.update_weights(0.5)
    torch.testing.assert_close(d.get_weights(), w0 - 0.5 * g)
    assert torch.equal(m[2].get_weights(), other)  # only this layer moves
