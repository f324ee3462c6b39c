"""GPU numerics of the training-support, image, recurrent and int8 kernels,
each against the plain-PyTorch / CPU-path oracle of the same op."""
import pytest
import torch

from dlvk_b200 import _ext
from dlvk_b200 import losses as Lo
from dlvk_b200 import optim as O
from dlvk_b200 import training as T
from dlvk_b200.data import transforms as TF
from dlvk_b200.models import layers as L
from dlvk_b200.models.sequential import Sequential

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def C():
    return _ext.C()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("probs", [False, True])
def test_step_metrics(dt, probs):
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(1000, 37, generator=g).to(DEV, dt)
    labels = torch.randint(0, 37, (1000,), generator=g, dtype=torch.int32).to(DEV)
    loss = torch.tensor([2.5], device=DEV)
    ls = torch.zeros(1, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int64, device=DEV)
    onehot = torch.nn.functional.one_hot(labels.long(), 37).float() if probs else None
    for _ in range(2):
        C().step_metrics(logits, None if probs else labels, onehot, loss, ls, cnt, 8.0)
    want = int((logits.float().argmax(-1) == labels.long()).sum()) * 2
    assert int(cnt) == want and float(ls) == pytest.approx(40.0)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_regularize_and_scale(dt):
    g = torch.Generator().manual_seed(1)
    w = torch.randn(10001, generator=g).to(DEV)
    w[::7] = 0
    gr = torch.randn(10001, generator=g).to(DEV, dt)
    ref = gr.float() + 4.0 * (0.01 * torch.sign(w) + 0.02 * w)
    loss = torch.zeros(1, device=DEV)
    k = torch.tensor([4.0], device=DEV)
    C().regularize(w, gr, 0.01, 0.02, 0.01, 0.0, loss, k)
    tol = 1e-6 if dt == torch.float32 else 2e-2
    assert torch.allclose(gr.float(), ref, atol=tol, rtol=tol)
    assert float(loss) == pytest.approx(float(0.01 * w.abs().sum()), rel=1e-4)
    x = torch.randn(777, generator=g).to(DEV, dt)
    x0 = x.float().clone()
    C().scale_by_device_scalar(x, k)
    assert torch.allclose(x.float(), x0 * 4.0, rtol=tol)


def test_grad_stats_device_scale_and_scaler_graph():
    """Loss-scaled training of a small bf16 MLP (scaler + regularizer inside
    the captured graph) tracks unscaled training."""
    g = torch.Generator().manual_seed(0)
    Cc = torch.randn(10, 32, generator=g) * 3
    y = torch.randint(0, 10, (512,), generator=g)
    x = Cc[y] + torch.randn(512, 32, generator=g)
    res = []
    for use in (False, True):
        m = Sequential(DEV, "fp32", seed=0)
        m.add_dense(32, 64).add_relu().add_dense(64, 10).add_softmax()
        m.build()
        opt = O.SGD(0.05)
        sc = T.GradientScaler(init_scale=2.0 ** 12, scale_window=4, device=DEV) if use else None
        st = T.TrainStep(m, Lo.CrossEntropyLoss(), opt, scaler=sc, regularizer=T.create_l2_regularization(1e-4),
                         metrics=True)
        for e in range(3):
            for i in range(0, 512, 128):
                st(x[i:i + 128].pin_memory(), y[i:i + 128].to(torch.int32).pin_memory())
        loss, acc, n = st.epoch_metrics()
        res.append((m.store.master.clone(), acc))
        if sc is not None:
            assert sc.get_scale() == 2.0 ** 15  # 12 clean steps, growth every 4
            assert st.graph is not None
        st.close()
    assert torch.allclose(res[0][0], res[1][0], rtol=1e-3, atol=1e-4)
    assert abs(res[0][1] - res[1][1]) < 0.02 and res[1][1] > 0.6


def test_scaler_overflow_skips_step_on_device():
    m = Sequential(DEV, "fp32", seed=0)
    m.add_dense(8, 4)
    m.build()
    opt = O.Adam(1e-2)
    sc = T.GradientScaler(init_scale=1024.0, device=DEV)
    m.store.grad.fill_(float("nan"))
    before = m.store.master.clone()
    sc.unscale_gradients(opt, m.store)
    opt.step(m)
    sc.update()
    torch.cuda.synchronize()
    assert sc.has_overflow() and sc.get_scale() == 512.0
    assert torch.equal(before, m.store.master)
    from dlvk_b200.ops.optim_kernels import read_hyper

    assert read_hyper(opt.state(m.store).hyper)["step"] == 0  # skipped step not counted


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_image_affine_sample(mode):
    g = torch.Generator().manual_seed(2)
    x = torch.rand(5, 3, 17, 23, generator=g)
    th = torch.randn(5, 6, generator=g) * 0.3
    th[:, 0] += 1
    th[:, 4] += 1
    th[:, 2] += 2
    th[:, 5] -= 1
    want = TF.affine_sample_reference(x, th, 19, 21, mode)
    got = C().image.affine_sample(x.to(DEV), th.to(DEV), 19, 21, mode, 0.0).cpu()
    bad = (got - want).abs() > 1e-5
    # nearest modes may differ only where the source coordinate sits on a
    # rounding boundary (fma vs separate mul/add in the two paths)
    assert bad.float().mean() < (0.002 if mode < 2 else 1e-9)


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_image_per_sample_stats(kind):
    g = torch.Generator().manual_seed(3)
    x = torch.rand(6, 3, 9, 11, generator=g)
    p = torch.rand(6, 2, generator=g) + torch.tensor([0.5, 1.0])
    want = TF.per_sample_stats_reference(x, kind, p, kind == 0)
    got = C().image.per_sample_stats(x.to(DEV), kind, p.to(DEV), kind == 0).cpu()
    assert torch.allclose(got, want, atol=2e-5)


def test_image_transforms_gpu_match_cpu():
    x = torch.rand(4, 3, 20, 20, generator=torch.Generator().manual_seed(4))
    for mk in (lambda: TF.RandomHorizontalFlip(0.5, seed=1), lambda: TF.RandomCrop(16, 16, 2, seed=2),
               lambda: TF.RandomBrightness(0.2, seed=3), lambda: TF.RandomContrast(0.3, seed=4),
               lambda: TF.Normalize([0.1, 0.2, 0.3], [0.5, 0.6, 0.7]), lambda: TF.Resize(13, 27),
               lambda: TF.Standardize(), lambda: TF.MinMaxScale(-1, 1), lambda: TF.CenterCrop(10, 12)):
        a, b = mk()(x), mk()(x.to(DEV)).cpu()
        assert torch.allclose(a, b, atol=2e-5), mk()
    nz = TF.RandomNoise(0.2, seed=0)(torch.zeros(8, 3, 64, 64, device=DEV))
    assert abs(float(nz.std()) - 0.2) < 0.005 and abs(float(nz.mean())) < 0.005


@pytest.mark.parametrize("cls", [L.RNNLayer, L.LSTMLayer, L.GRULayer])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_recurrent_gpu_vs_cpu(cls, dt):
    torch.manual_seed(0)
    cpu = cls(64, 64)
    gpu = cpu.clone()
    cpu.to("cpu", torch.float32)
    gpu.to(DEV, dt)
    x = torch.randn(16, 12, 64)
    gy = torch.randn(16, 12, 64)
    yc = cpu.forward(x)
    dxc = cpu.backward(gy)
    yg = gpu.forward(x.to(DEV, dt))
    dxg = gpu.backward(gy.to(DEV, dt))
    tol = 2e-3 if dt == torch.float32 else 6e-2
    assert torch.allclose(yg.float().cpu(), yc, atol=tol, rtol=tol)
    assert torch.allclose(dxg.float().cpu(), dxc, atol=tol * 2, rtol=tol)
    for pc, pg in zip(cpu.parameters(), gpu.parameters()):
        scale = pc.grad.abs().max().item() + 1e-6
        assert (pg.grad.cpu() - pc.grad).abs().max().item() / scale < tol * 2, pc.name


def test_bidirectional_lstm_gpu():
    torch.manual_seed(1)
    cpu = L.BidirectionalRNN("lstm", 32, 32)
    gpu = cpu.clone()
    cpu.to("cpu", torch.float32)
    gpu.to(DEV, torch.float32)
    x = torch.randn(8, 10, 32)
    g = torch.randn(8, 10, 64)
    yc, yg = cpu.forward(x), gpu.forward(x.to(DEV))
    dc, dg = cpu.backward(g), gpu.backward(g.to(DEV))
    assert torch.allclose(yg.cpu(), yc, atol=2e-3) and torch.allclose(dg.cpu(), dc, atol=4e-3)


@pytest.mark.parametrize("shape", [(256, 512, 384), (100, 96, 200), (1024, 1024, 2048)])
@pytest.mark.parametrize("path", [1, 2])
def test_int8_gemm(shape, path):
    M, K, N = shape
    g = torch.Generator().manual_seed(5)
    a = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g)
    bias = torch.randn(N, generator=g)
    from dlvk_b200.ops import quant as Q

    qa, sa = Q.quantize_rows(a)
    qw, sw = Q.quantize_rows(w)
    qa_g, sa_g = Q.quantize_rows(a.to(DEV))
    # the device quantiser may round the other way exactly at .5 boundaries
    d = (qa_g.cpu().int() - qa.int()).abs()
    assert d.max() <= 1 and (d > 0).float().mean() < 1e-4 and torch.allclose(sa_g.cpu(), sa)
    want = Q.gemm_i8(qa_g.cpu(), qw, sa_g.cpu(), sw, bias, 1)
    got = C().gemm_i8(qa_g, qw.to(DEV), sa_g, sw.to(DEV), bias.to(DEV), 1, None, path)
    assert torch.allclose(got.float().cpu(), want, rtol=1e-4, atol=1e-3)
    deq = torch.relu(a @ w.t() + bias)
    assert ((got.float().cpu() - deq).abs().max() / deq.abs().max()) < 0.03


def test_quantized_model_matches_fp32():
    from dlvk_b200.optimization.model_optimizer import ModelOptimizer

    m = Sequential(DEV, "fp32", seed=0)
    m.add_dense(256, 512).add_relu().add_dense(512, 10)
    m.build()
    m.set_training(False)
    x = torch.randn(128, 256, device=DEV)
    y = m.forward(x)
    opt = ModelOptimizer(m)
    qm = opt.quantize_model()
    yq = qm.forward(x)
    assert ((yq.float() - y.float()).abs().max() / y.abs().max()) < 0.05
    assert opt.stats.compression_ratio > 3.0


def test_dataloader_to_device_prefetch():
    from dlvk_b200.data import DataLoader, MnistDataset

    ds = MnistDataset("/nonexistent")
    dl = DataLoader(ds, DEV, batch_size=128, shuffle=True, one_hot=False, prefetch=3,
                    batch_transform=TF.Normalize([0.1307], [0.3081]))
    n = 0
    for bx, by in dl:
        assert bx.is_cuda and by.dtype == torch.int32 and bx.shape[1:] == (1, 28, 28)
        n += bx.shape[0]
    assert n == 1000 and dl.h2d_bytes > 0
    ref = DataLoader(ds, None, batch_size=128, shuffle=True, one_hot=False)
    bx0 = next(iter(ref))[0]
    bxg = next(iter(dl))[0]
    assert torch.allclose(bxg.cpu(), (bx0 - 0.1307) / 0.3081, atol=1e-5)


def test_trainer_gpu_end_to_end():
    from dlvk_b200.data import DataLoader, TensorDataset

    g = torch.Generator().manual_seed(0)
    Cc = torch.randn(10, 32, generator=g) * 3
    y = torch.randint(0, 10, (1024,), generator=g)
    x = Cc[y] + torch.randn(1024, 32, generator=g)
    ds = TensorDataset(x, y.to(torch.int32), 10)
    dl = DataLoader(ds, DEV, batch_size=128, one_hot=False)
    m = Sequential(DEV, "bf16", seed=0)
    m.add_dense(32, 128).add_relu().add_dense(128, 10).add_softmax()
    trn = T.create_trainer(m, "adam", 3e-3, "crossentropy")
    hist = trn.fit(dl, dl, epochs=3, verbose=False)
    assert hist[-1].accuracy > 0.9 and hist[-1].val_accuracy > 0.9
    trn.close()
