"""Recurrent layers against torch.nn (CPU oracle) and model export
round-trips (DLVK, ONNX, GGUF v3, SafeTensors), with the third-party
safetensors / gguf readers as independent checks where installed."""
import importlib.util
import os

import pytest
import torch

from dlvk_b200.export import ModelExportManager, ModelFormat, ModelMetadata
from dlvk_b200.export import onnx as ox
from dlvk_b200.models import layers as L
from dlvk_b200.models.sequential import Sequential

REF = {"RNN": torch.nn.RNN, "LSTM": torch.nn.LSTM, "GRU": torch.nn.GRU}


def _copy(ref, cells):
    with torch.no_grad():
        for sfx, c in zip(["", "_reverse"], cells):
            getattr(ref, "weight_ih_l0" + sfx).copy_(c.w_ih.master)
            getattr(ref, "weight_hh_l0" + sfx).copy_(c.w_hh.master)
            getattr(ref, "bias_ih_l0" + sfx).copy_(c.b_ih.master)
            getattr(ref, "bias_hh_l0" + sfx).copy_(c.b_hh.master)


@pytest.mark.parametrize("cls", [L.RNNLayer, L.LSTMLayer, L.GRULayer])
def test_recurrent_vs_torch(cls):
    torch.manual_seed(0)
    lay = cls(5, 8).to("cpu", torch.float32)
    x = torch.randn(3, 7, 5)
    y = lay.forward(x)
    g = torch.randn_like(y)
    dx = lay.backward(g)
    ref = REF[lay.type_name](5, 8, batch_first=True)
    _copy(ref, [lay])
    xr = x.clone().requires_grad_(True)
    yr, _ = ref(xr)
    yr.backward(g)
    assert torch.allclose(y, yr, atol=1e-5)
    assert torch.allclose(dx, xr.grad, atol=1e-5)
    assert torch.allclose(lay.w_ih.grad, ref.weight_ih_l0.grad, atol=1e-5)
    assert torch.allclose(lay.w_hh.grad, ref.weight_hh_l0.grad, atol=1e-5)
    assert torch.allclose(lay.b_ih.grad, ref.bias_ih_l0.grad, atol=1e-5)
    assert torch.allclose(lay.b_hh.grad, ref.bias_hh_l0.grad, atol=1e-5)


@pytest.mark.parametrize("cell", ["rnn", "lstm", "gru"])
def test_bidirectional_vs_torch(cell):
    torch.manual_seed(1)
    bl = L.BidirectionalRNN(cell, 4, 6).to("cpu", torch.float32)
    x = torch.randn(2, 5, 4)
    y = bl.forward(x)
    g = torch.randn_like(y)
    dx = bl.backward(g)
    ref = REF[cell.upper()](4, 6, batch_first=True, bidirectional=True)
    _copy(ref, [bl.fwd, bl.bwd])
    xr = x.clone().requires_grad_(True)
    yr, _ = ref(xr)
    yr.backward(g)
    assert torch.allclose(y, yr, atol=1e-5) and torch.allclose(dx, xr.grad, atol=1e-5)
    assert torch.allclose(bl.bwd.w_hh.grad, ref.weight_hh_l0_reverse.grad, atol=1e-5)


def test_lstm_forget_bias_and_states():
    lay = L.LSTMLayer(3, 4).to("cpu", torch.float32)
    b = lay.b_ih.master
    assert torch.all(b[4:8] == 1) and torch.all(b[:4] == 0) and torch.all(b[8:] == 0)
    x = torch.randn(2, 3, 3)
    lay.set_states(torch.ones(2, 4), torch.ones(2, 4))
    y1 = lay.forward(x)
    lay.reset_states()
    y0 = lay.forward(x)
    assert not torch.allclose(y1, y0)
    assert torch.equal(lay.get_hidden_state(), y0[:, -1])


def _models():
    torch.manual_seed(0)
    mlp = Sequential("cpu", "fp32", seed=0)
    mlp.add_dense(12, 16).add_relu().add_batchnorm1d(16).add_dropout(0.1).add_dense(16, 5).add_softmax()
    mlp.build()
    mlp.forward(torch.randn(8, 12))  # move the running statistics
    cnn = Sequential("cpu", "fp32", seed=0)
    cnn.add_conv2d(3, 4, 3, 1, 1).add_relu().add_maxpool2d(2).add_avgpool2d(2).add_flatten().add_dense(16, 3)
    cnn.build()
    rnn = Sequential("cpu", "fp32", seed=0)
    rnn.add_lstm(6, 8).add_bidirectional("gru", 8, 5).add_dense(10, 3)
    rnn.build()
    tfm = Sequential("cpu", "fp32", seed=0)
    tfm.add_embedding(50, 16).add_positional_encoding(16, 64).add_transformer_encoder(16, 2, 32)
    tfm.add_layernorm(16).add_dense(16, 50)
    tfm.build()
    with torch.no_grad():
        for p in tfm.parameters():
            p.master.add_(0.05 * torch.randn_like(p.master))
    tfm.store.sync_value()
    return [("mlp", mlp, torch.randn(4, 12), [4, 12]), ("cnn", cnn, torch.randn(2, 3, 8, 8), [2, 3, 8, 8]),
            ("rnn", rnn, torch.randn(2, 4, 6), [2, 4, 6]),
            ("transformer", tfm, torch.randint(0, 50, (2, 6), dtype=torch.int32), [2, 6])]


@pytest.mark.parametrize("case", range(4))
def test_export_roundtrip_all_formats(tmp_path, case):
    name, m, x, shape = _models()[case]
    M = ModelExportManager()
    m.set_training(False)
    y = m.forward(x)
    for fmt in M.get_supported_formats():
        p = str(tmp_path / ("m" + M.get_extension(fmt)))
        kw = {"input_shape": shape} if fmt is ModelFormat.ONNX else {}
        assert M.export_model(m, p, fmt, ModelMetadata(name=name, hidden_size=7, custom_metadata={"k": "v"}), **kw)
        assert M.detect_format(p) is fmt
        m2, md = M.import_model(p, device="cpu")
        m2.set_training(False)
        assert torch.equal(m2.forward(x), y), fmt
        assert md.name == name and md.hidden_size == 7
        if fmt is ModelFormat.ONNX:
            parsed = ox.parse_model(open(p, "rb").read())
            assert parsed["opset"] == 17 and parsed["ir_version"] == 8
            yo = ox.run(parsed, x if x.is_floating_point() else x.long())
            assert torch.allclose(yo, y, atol=1e-5)


@pytest.mark.skipif(importlib.util.find_spec("safetensors") is None, reason="safetensors not installed")
def test_safetensors_readable_by_library(tmp_path):
    import safetensors.torch as st

    name, m, x, _ = _models()[0]
    p = str(tmp_path / "m.safetensors")
    ModelExportManager().export_model(m, p, ModelFormat.SAFETENSORS)
    ref = st.load_file(p)
    for n, t in m.state_tensors():
        assert torch.equal(ref[n], t)


@pytest.mark.skipif(importlib.util.find_spec("gguf") is None, reason="gguf not installed")
def test_gguf_readable_by_library(tmp_path):
    import gguf
    import numpy as np

    name, m, x, _ = _models()[2]
    p = str(tmp_path / "m.gguf")
    ModelExportManager().export_model(m, p, ModelFormat.GGUF, ModelMetadata(name="rnn"))
    r = gguf.GGUFReader(p)
    by = {t.name: t for t in r.tensors}
    for n, t in m.state_tensors():
        got = np.asarray(by[n].data).reshape(tuple(t.shape))
        assert np.array_equal(got, t.numpy())
    f = r.fields["general.name"]
    assert bytes(f.parts[f.data[0]]).decode() == "rnn"


def test_hdf5_reports_missing_dependency(tmp_path):
    if importlib.util.find_spec("h5py") is not None:
        pytest.skip("h5py installed")
    with pytest.raises(RuntimeError, match="h5py"):
        ModelExportManager().export_model(_models()[0][1], str(tmp_path / "m.h5"), ModelFormat.HDF5)
