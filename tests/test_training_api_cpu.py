"""CPU tests of the training API: ModelTrainer / Trainer / AdvancedTrainer,
callbacks, loss scaling, regularisation, schedulers, search, persistence."""
import io
import math
import os

import pytest
import torch

from dlvk_b200 import losses as Lo
from dlvk_b200 import optim as O
from dlvk_b200 import training as T
from dlvk_b200.data import DataLoader, TensorDataset
from dlvk_b200.models.sequential import Sequential


def clusters(n=400, d=20, k=10, seed=0):
    g = torch.Generator().manual_seed(seed)
    C = torch.randn(k, d, generator=g) * 3
    y = torch.randint(0, k, (n,), generator=g)
    return C[y] + torch.randn(n, d, generator=g), y


def mlp(d=20, k=10):
    m = Sequential("cpu", "fp32", seed=0)
    m.add_dense(d, 32).add_relu().add_dense(32, k).add_softmax()
    return m.build()


def test_model_trainer_fit_evaluate_predict(tmp_path):
    x, y = clusters()
    m = mlp()
    tr = T.ModelTrainer(m)
    tr.compile(O.Adam(3e-3), Lo.CrossEntropyLoss())
    csv = tmp_path / "log.csv"
    tr.add_callback(T.CSVLogger(str(csv)))
    ck = T.ModelCheckpoint(str(tmp_path / "best.dlvk"), monitor="val_loss")
    tr.add_callback(ck)
    hist = tr.fit(x, y, epochs=6, batch_size=50, validation_split=0.25, verbose=False)
    assert hist[-1].loss < hist[0].loss
    assert hist[-1].validation_accuracy > 0.9
    assert csv.read_text().count("\n") == 7
    assert ck.saved and os.path.exists(ck.saved[-1])
    ev = tr.evaluate(x, y, 100)
    assert ev.accuracy > 0.9
    p = tr.predict(x[:7], batch_size=3)
    assert p.shape == (7, 10)
    assert torch.allclose(p.sum(-1), torch.ones(7), atol=1e-5)


def test_trainer_with_dataloader_and_callbacks():
    x, y = clusters()
    ds = TensorDataset(x, y.to(torch.int32), 10)
    dl = DataLoader(ds, None, batch_size=40, shuffle=True, one_hot=True)
    vl = DataLoader(TensorDataset(*clusters(100, seed=0)), None, batch_size=50, shuffle=False, one_hot=False)
    trn = T.create_trainer(mlp(), "adam", 5e-3, "crossentropy")
    buf = io.StringIO()
    trn.add_callback(T.ProgressCallback(5, stream=buf))
    trn.add_callback(T.ReduceLROnPlateau("loss", factor=0.5, patience=100))
    hist = trn.fit(dl, vl, epochs=5, verbose=False)
    assert len(hist) == 5 and hist[-1].accuracy > 0.9 and hist[-1].val_accuracy > 0.9
    assert "Epoch 5/5" in buf.getvalue()
    assert all(h.samples_per_s > 0 for h in hist)


def test_early_stopping_stops_and_restores():
    es = T.EarlyStopping("val_loss", patience=2)
    tr = type("Tr", (), {"stop_training": False})()
    es.trainer = tr
    es.on_train_begin()
    for e, v in enumerate([1.0, 0.9, 0.95, 0.96]):
        es.on_epoch_end(e, T.TrainingMetrics(validation_loss=v))
    assert es.should_stop() and tr.stop_training and es.stopped_epoch == 3


@pytest.mark.parametrize("opt", ["sgd", "adam"])
def test_scaler_matches_unscaled_training(opt):
    """Loss scaling with unscale-in-optimizer must not change the trajectory."""
    x, y = clusters(200)
    res = []
    for use in (False, True):
        m = mlp()
        o = T.make_optimizer(opt, 0.05 if opt == "sgd" else 3e-3)
        sc = T.GradientScaler(init_scale=2.0 ** 10, scale_window=3, device="cpu") if use else None
        st = T.TrainStep(m, Lo.CrossEntropyLoss(), o, scaler=sc, metrics=True)
        for i in range(0, 200, 50):
            st(x[i:i + 50], y[i:i + 50])
        res.append(m.store.master.clone())
    assert torch.allclose(res[0], res[1], rtol=1e-4, atol=1e-5)


def test_scaler_backoff_and_growth():
    sc = T.GradientScaler(init_scale=1024.0, scale_window=2, device="cpu")
    m = mlp()
    o = O.SGD(0.1)
    m.store.grad.fill_(float("inf"))
    before = m.store.master.clone()
    sc.unscale_gradients(o, m.store)
    assert sc.has_overflow()
    o.step(m)
    sc.update()
    assert sc.get_scale() == 512.0 and torch.equal(before, m.store.master)  # step skipped
    m.store.grad.fill_(1.0)
    for _ in range(2):
        sc.unscale_gradients(o, m.store)
        o.step(m)
        sc.update()
    assert sc.get_scale() == 1024.0
    sc.load_state_dict({"scale": 65536.0 * 4})
    assert sc.state_dict()["scale"] == 262144.0


def test_regularizers_math():
    w = torch.tensor([[1.0, -2.0], [0.0, 3.0]])
    l1, l2 = T.L1Regularizer(0.1), T.L2Regularizer(0.2)
    assert math.isclose(l1.compute_loss([w]), 0.1 * 6.0, rel_tol=1e-6)
    assert math.isclose(l2.compute_loss([w]), 0.5 * 0.2 * 14.0, rel_tol=1e-6)
    assert torch.allclose(l1.compute_gradients([w])[0], 0.1 * torch.sign(w))
    en = T.ElasticNetRegularizer(0.2, 0.25)
    assert en.coefficients() == pytest.approx((0.05, 0.15))
    wd = T.WeightDecayRegularizer(0.01)
    assert wd.compute_loss([w]) == 0.0
    ww = w.clone()
    wd.apply_decay([ww], 0.5)
    assert torch.allclose(ww, w * (1 - 0.005))
    mgr = T.create_comprehensive_regularization(0.01, 0.001, True, 0.002)
    assert mgr.size() == 3
    stats = mgr.get_stats([w])
    assert stats["regularizer_names"] == ["L2", "WeightDecay", "L1"]
    assert math.isclose(stats["total_loss"], mgr.compute_total_loss([w]), rel_tol=1e-6)


def test_regularization_manager_fused_store_path():
    m = mlp()
    m.store.grad.zero_()
    mgr = T.create_elastic_net(0.1, 0.5)
    loss = mgr.apply_to_store(m.store)
    ws = [p for p in m.parameters() if p.decay]
    want = sum(0.05 * p.master.abs().sum() + 0.5 * 0.05 * (p.master ** 2).sum() for p in ws)
    assert torch.allclose(loss, want.reshape(1), rtol=1e-5)
    for p in m.parameters():
        exp = (0.05 * torch.sign(p.master) + 0.05 * p.master) if p.decay else torch.zeros_like(p.master)
        assert torch.allclose(p.grad, exp, atol=1e-7)


def test_advanced_dropout_schedule():
    ad = T.AdvancedDropout(0.5, warmup_epochs=4, adaptive=True)
    ad.update_rate(2)
    assert ad.get_current_rate() == pytest.approx(0.25)
    ad.update_rate(4, 1.0)
    ad.update_rate(5, 1.2)
    assert ad.get_current_rate() == pytest.approx(0.275)  # x1.1 of the warm-up rate left at epoch 2


def test_schedulers():
    c = T.CosineAnnealingScheduler(1.0, 0.0, 10)
    assert c.get_lr(0, 1.0) == pytest.approx(1.0)
    for _ in range(5):
        c.step()
    assert c.get_lr(0, 1.0) == pytest.approx(0.5)
    oc = T.OneCycleScheduler(1.0, 10, 0.1, 0.01, 30)
    vals = []
    for _ in range(11):
        vals.append(oc.get_lr(0, 0))
        oc.step()
    assert vals[0] == pytest.approx(0.1) and max(vals) == pytest.approx(1.0) and vals[-1] == pytest.approx(0.01)
    rp = T.ReduceOnPlateauScheduler(0.5, patience=2)
    lr = 1.0
    for v in [1.0, 0.5, 0.6, 0.6, 0.6]:
        lr = rp.get_lr(0, lr, v)
    assert lr == 0.5


def test_advanced_trainer(tmp_path):
    x, y = clusters()
    dl = DataLoader(TensorDataset(x, y.to(torch.int32), 10), None, batch_size=50, one_hot=False)
    cfg = T.AdvancedTrainingConfig(use_regularization=True, l2_lambda=1e-4, use_gradient_clipping=True,
                                   lr_schedule=T.LRScheduleType.COSINE_ANNEALING, checkpoint_dir=str(tmp_path),
                                   verbose_training=False, use_mixed_precision=True)
    at = T.create_advanced_trainer(mlp(), "adam", 5e-3, "crossentropy", cfg)
    hist = at.fit(dl, dl, 4)
    assert hist[-1].val_accuracy > 0.9
    st = at.get_statistics()
    assert st.total_epochs_trained == 4 and st.final_l2_loss > 0
    assert (tmp_path / "best_model.dlvk").exists() and (tmp_path / "training_curves.json").exists()


def test_random_search():
    cfg = T.HyperparameterConfig({"lr": T.HyperparameterRange(1e-4, 1e-1, True),
                                  "wd": T.HyperparameterRange(0.0, 1.0)}, n_trials=60)
    r = T.random_search(lambda p: (math.log10(p["lr"]) + 2) ** 2 + p["wd"], cfg)
    assert abs(math.log10(r.best_params["lr"]) + 2) < 0.5 and len(r.all_results) == 60


def test_persistence(tmp_path):
    m = mlp()
    x, _ = clusters(8)
    ck = T.CheckpointManager(str(tmp_path), "mlp", save_best_only=False, max_checkpoints=2)
    opt = O.Adam(1e-3)
    for e in range(4):
        ck.save_checkpoint(m, T.TrainingMetrics(loss=1.0 / (e + 1), validation_loss=1.0 / (e + 1)), e, opt)
    names = [os.path.basename(p) for p in ck.list_checkpoints()]
    assert names == ["mlp_epoch_0002.dlvk", "mlp_epoch_0003.dlvk"]
    mm, data = ck.load_checkpoint(ck.get_best_checkpoint_path())
    assert data.current_epoch == 3 and data.current_metrics.loss == pytest.approx(0.25)
    assert torch.equal(mm.forward(x), m.forward(x))
    ver = T.ModelVersioning(str(tmp_path / "exp"))
    ver.create_experiment("e1")
    ver.save_model_version(m, metrics={"val_loss": 0.5})
    ver.save_model_version(mlp(), metrics={"val_loss": 0.4})
    assert ver.list_versions() == ["v001", "v002"]
    assert ver.compare_versions("v001", "v002")["better_version"] == "v002"
    assert torch.equal(ver.load_model_version("v001").forward(x), m.forward(x))
    ser = T.ModelSerializer(T.SerializationFormat.DLVK_JSON)
    ser.save(m, str(tmp_path / "m.json"))
    assert torch.equal(ser.load(str(tmp_path / "m.json")).forward(x), m.forward(x))


def test_overlapped_update_matches_step_after_backward():
    """Per-bucket updates driven by the grad-ready hooks give the same weights
    as one optimizer step after backward."""
    from dlvk_b200.training.overlap import OverlappedUpdate
    from dlvk_b200.training.step import TrainStep

    x, y = clusters(64)
    y = y.to(torch.int32)
    ma, mb = mlp(), mlp()
    ov = OverlappedUpdate(mb, O.Adam(1e-2), bucket_mb=0.001)
    assert len(ov.buckets) > 1
    sa = TrainStep(ma, Lo.CrossEntropyLoss(), O.Adam(1e-2))
    sb = TrainStep(mb, Lo.CrossEntropyLoss(), ov.opt, dp=ov)
    for _ in range(4):
        la, lb = sa(x, y), sb(x, y)
    assert torch.allclose(torch.as_tensor(la), torch.as_tensor(lb), atol=1e-6)
    assert torch.allclose(ma.store.master, mb.store.master, atol=1e-6)
    ov.close()
    clipped = O.Adam(1e-2)
    clipped.set_gradient_clipping(max_norm=1.0)
    with pytest.raises(ValueError):
        OverlappedUpdate(mlp(), clipped)
