"""CPU tests: the framework's reference path against the C++ oracle and
against plain PyTorch autograd; .dlvk persistence."""
import io
import math
import struct

import pytest
import torch
import torch.nn.functional as F

import dlvk_b200 as dl
from dlvk_b200 import _ext
from dlvk_b200.models import zoo

C = _ext.C()


def close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= tol * (b.abs().max().item() + 1e-6) + 1e-7, err


def test_mlp_config1_matches_oracle():
    """Config 1: Dense 784->128, ReLU, Dense 128->10, softmax, CE, one Adam step."""
    m = zoo.mlp(device="cpu", seed=0)
    m.build()
    x, y = zoo.synthetic_batch("mlp", 32, seed=0)
    W1 = m[0].weight.master.clone()
    b1 = m[0].bias.master.clone()
    W2 = m[2].weight.master.clone()
    b2 = m[2].bias.master.clone()
    # oracle forward
    h = C.ref.relu(C.ref.dense_fwd(x, W1, b1))
    logits = C.ref.dense_fwd(h, W2, b2)
    p = C.ref.softmax(logits)
    t = torch.zeros(32, 10)
    t[torch.arange(32), y.long()] = 1
    loss_ref = C.ref.cross_entropy(p, t)
    # framework forward
    m.set_training(False)
    out = m.forward(x)
    close(out, p, 1e-5)
    m.set_training(True)
    opt = dl.Adam(1e-3)
    loss = m.train_step(x, y, dl.CrossEntropyLoss(), opt)
    assert abs(float(loss) - loss_ref) < 1e-4
    # oracle backward: grad wrt logits (p - t)/B through the identity softmax-bwd
    g = C.ref.cross_entropy_grad(p, t)
    dh, dW2, db2 = C.ref.dense_bwd(h, W2, g)
    dh = C.ref.relu_bwd(dh, C.ref.dense_fwd(x, W1, b1))
    _, dW1, db1 = C.ref.dense_bwd(x, W1, dh)
    close(m[2].weight.grad, dW2, 1e-5)
    close(m[2].bias.grad, db2, 1e-5)
    close(m[0].weight.grad, dW1, 1e-5)
    close(m[0].bias.grad, db1, 1e-5)
    # oracle Adam step (bias-corrected, step 1)
    for P, G, got in ((W1, dW1, m[0].weight.master), (b2, db2, m[2].bias.master)):
        mm, vv = torch.zeros_like(P), torch.zeros_like(P)
        C.ref.adam(P, G.contiguous(), mm, vv, 1e-3, 0.9, 0.999, 1e-8, 1, True)
        close(got, P, 1e-5)


def test_dlvk_v2_roundtrip_bit_exact(tmp_path):
    m = zoo.small_cnn(device="cpu", seed=3)
    opt = dl.Adam(1e-3)
    x, y = zoo.synthetic_batch("cnn", 8)
    m.train_step(x, y, dl.CrossEntropyLoss(), opt)
    a, b = tmp_path / "a.dlvk", tmp_path / "b.dlvk"
    m.save_weights(str(a), optimizer=opt)
    m2 = zoo.small_cnn(device="cpu", seed=4)
    opt2 = dl.Adam(1e-3)
    m2.load_weights(str(a), optimizer=opt2)
    m2.save_weights(str(b), optimizer=opt2)
    assert a.read_bytes() == b.read_bytes()
    l1 = m.train_step(x, y, dl.CrossEntropyLoss(), opt)
    l2 = m2.train_step(x, y, dl.CrossEntropyLoss(), opt2)
    assert float(l1) == float(l2)
    assert torch.equal(m.store.master, m2.store.master)


def test_dlvk_v2_layout():
    blob = C.io.encode_v2('{"k":1}', [("w", 0, [2, 3], bytes(range(24)))])
    assert blob[:4] == b"DLVK"
    assert struct.unpack("<II", blob[4:12]) == (2, 7)
    assert blob[12:19] == b'{"k":1}'
    n = struct.unpack("<I", blob[19:23])[0]
    assert n == 1
    off = blob.index(bytes(range(24)))
    assert off % 64 == 0
    v, variant, meta, recs = C.io.decode(blob)
    assert (v, variant, meta) == (2, "v2", '{"k":1}')
    assert recs[0][0] == "w" and list(recs[0][2]) == [2, 3] and recs[0][3] == bytes(range(24))


# The reference's 77-byte weight-bearing v1 sample (a 1->1 linear model with
# w = 25.6, b = 8.7, activation "linear", loss 60.375, 12 epochs).
V1_SAMPLE = bytes.fromhex(
    "444c564b01000000020000000100000001000000010000" "00cdcccc410100000033330b41060000006c696e656172"
    "008071420c00000013000000323032352d30372d32342031303a32323a3230")


def test_dlvk_v1_weight_reader(tmp_path):
    p = tmp_path / "linear_model.dlvk"
    p.write_bytes(V1_SAMPLE)
    assert len(V1_SAMPLE) == 77
    from dlvk_b200.utils import dlvk_io

    version, variant, meta, tens = dlvk_io.load(str(p))
    assert version == 1 and variant == "v1-weights"
    assert meta["activation"] == "linear" and meta["epochs_trained"] == 12
    assert abs(meta["final_loss"] - 60.375) < 1e-6
    assert abs(float(tens["weights"][0]) - 25.6) < 1e-5 and abs(float(tens["biases"][0]) - 8.7) < 1e-5
    m = dl.Sequential("cpu")
    m.add_dense(1, 1)
    m.load_weights(str(p))
    m.set_training(False)
    assert abs(float(m.forward(torch.tensor([[2.0]]))[0, 0]) - (2 * 25.6 + 8.7)) < 1e-4


def test_dlvk_v1_header_reader():
    blob = C.io.encode_v1_header('{"name":"m"}')
    v, variant, meta, recs = C.io.decode(blob)
    assert v == 1 and variant == "v1-header" and meta == '{"name":"m"}' and len(recs) == 0


def test_truncated_file_raises(tmp_path):
    p = tmp_path / "t.dlvk"
    blob = C.io.encode_v2("{}", [("w", 0, [4], b"\0" * 16)])
    p.write_bytes(blob[:-5])
    with pytest.raises(Exception):
        C.io.load(str(p))


def _torch_block(x, blk):
    """Plain autograd reference of one pre-norm encoder block."""
    B, S, E = x.shape
    H, D = blk.attn.num_heads, blk.attn.head_dim
    P = {id(p): p.master.clone().requires_grad_(True) for p in blk.parameters()}
    g = lambda p: P[id(p)]
    h1 = F.layer_norm(x, (E,), g(blk.ln1.gamma), g(blk.ln1.beta), 1e-5)
    qkv = (h1 @ g(blk.attn.w_qkv)).reshape(B, S, 3, H, D)
    q, k, v = qkv[:, :, 0].transpose(1, 2), qkv[:, :, 1].transpose(1, 2), qkv[:, :, 2].transpose(1, 2)
    a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, S, E)
    h = a @ g(blk.attn.w_o) + x
    h2 = F.layer_norm(h, (E,), g(blk.ln2.gamma), g(blk.ln2.beta), 1e-5)
    f = torch.relu(h2 @ g(blk.ff1.weight) + g(blk.ff1.bias))
    y = f @ g(blk.ff2.weight) + g(blk.ff2.bias) + h
    return y, P


def test_transformer_block_fused_backward_matches_autograd():
    torch.manual_seed(0)
    blk = dl.TransformerEncoderLayer(64, 4, 128, init_std=0.1).to("cpu")
    x = torch.randn(2, 16, 64)
    xr = x.clone().requires_grad_(True)
    yr, P = _torch_block(xr, blk)
    gy = torch.randn_like(yr)
    yr.backward(gy)
    xs = x.clone().requires_grad_(True)
    blk._store.zero_grad()
    y = blk.forward(xs)
    close(y, yr.detach(), 1e-5)
    (dx,) = torch.autograd.grad(y, xs, gy)
    close(dx, xr.grad, 1e-4)
    for p in blk.parameters():
        close(p.grad, P[id(p)].grad, 1e-4)


def test_layer_cpu_paths_match_torch():
    from dlvk_b200.ops import nn as NN

    x = torch.randn(2, 3, 8, 8)
    w = torch.randn(4, 3, 3, 3)
    close(NN.conv2d_fwd(x, w, None, 1, 1), F.conv2d(x, w, padding=1), 1e-6)
    close(NN.avgpool_fwd(x, 3, 2, 1), F.avg_pool2d(x, 3, 2, 1, count_include_pad=False), 1e-6)
    y, idx = NN.maxpool_fwd(x, 2, 2)
    close(y, F.max_pool2d(x, 2, 2), 0)
    # oracle conv agrees with torch
    close(C.ref.conv2d_fwd(x.contiguous(), w.contiguous(), None, 1, 1), F.conv2d(x, w, padding=1), 1e-5)
    dx, dw, db = C.ref.conv2d_bwd(x.contiguous(), w.contiguous(), torch.ones(2, 4, 8, 8), 1, 1)
    close(dw, torch.nn.grad.conv2d_weight(x, w.shape, torch.ones(2, 4, 8, 8), padding=1), 1e-5)


def test_dropout_is_reproducible_and_unbiased():
    keep = C.ref.dropout_mask(100000, 0.1, 42, 1, 0).float()
    assert abs(keep.mean().item() - 0.9) < 0.01
    assert torch.equal(keep, C.ref.dropout_mask(100000, 0.1, 42, 1, 0).float())
    assert not torch.equal(keep, C.ref.dropout_mask(100000, 0.1, 42, 1, 1).float())


def test_optimizers_cpu_match_oracle():
    for opt, ref in ((dl.SGD(0.1, 0.9), "sgd"), (dl.RMSprop(0.01), "rmsprop"), (dl.Adam(1e-2), "adam")):
        m = dl.Sequential("cpu", seed=1)
        m.add_dense(16, 8)
        m.build()
        P = m.store.master.clone()
        m.store.grad.copy_(torch.randn_like(P))
        G = m.store.grad.clone()
        opt.step(m)
        s1, s2 = torch.zeros_like(P), torch.zeros_like(P)
        if ref == "sgd":
            C.ref.sgd(P, G, s1, 0.1, 0.9)
        elif ref == "rmsprop":
            C.ref.rmsprop(P, G, s1, 0.01, 0.99, 1e-8)
        else:
            C.ref.adam(P, G, s1, s2, 1e-2, 0.9, 0.999, 1e-8, 1, True)
        close(m.store.master, P, 1e-6)


def test_sequential_api_surface():
    m = dl.Sequential("cpu")
    m.add_conv2d(1, 2, 3, 1, 1)
    m.add_batchnorm2d(2)
    m.add_relu()
    m.add_avgpool2d(2)
    m.add_flatten()
    m.add_dense(2 * 4 * 4, 5)
    m.add_sigmoid()
    m.add_dense(5, 3)
    m.add_tanh()
    m.add_dropout(0.2)
    m.add_dense(3, 2)
    m.add_softmax()
    y = m.forward(torch.randn(4, 1, 8, 8))
    assert y.shape == (4, 2)
    assert "Total params" in m.summary()
    assert m.parameter_count() == sum(p.numel for p in m.parameters())
    c = m.clone()
    assert c.size() == m.size()
    loss = m.train_step(torch.randn(4, 1, 8, 8), torch.tensor([0, 1, 1, 0], dtype=torch.int32),
                        dl.CrossEntropyLoss(), dl.SGD(0.1, 0.9))
    assert math.isfinite(float(loss))


def test_tensor_facade_ops():
    t = dl.Tensor([2, 3], device="cpu")
    t.upload_data([[1, 2, 3], [4, 5, 6]])
    assert t.sum(0).download_data().tolist() == [5, 7, 9]
    assert t.transpose().shape() == [3, 2]
    r = dl.Tensor([2, 3], device="cpu")
    assert dl.TensorOpsStatic.relu(t.multiply_scalar(-1.0), r)
    assert float(r.data.abs().sum()) == 0.0
    d = t.divide(dl.Tensor([2, 3], device="cpu"))
    assert float(d.data[0, 0]) == 1e8


def test_relu_bitmask_pack_roundtrip_cpu():
    """The CPU restatement of the GEMM's ReLU bitmask: pack / unpack round trip
    and the forward / backward pair against a plain mask."""
    import torch
    from dlvk_b200.ops import core as K

    g = torch.Generator().manual_seed(3)
    for m, n in ((5, 32), (7, 45), (3, 100)):
        pos = torch.rand(m, n, generator=g) > 0.5
        bits = K._pack_bits(pos, (n + 31) // 32)
        assert bits.dtype == torch.int32 and bits.shape == (m, (n + 31) // 32)
        assert torch.equal(K._unpack_bits(bits, n), pos)
    a, b = torch.randn(6, 8, generator=g), torch.randn(8, 40, generator=g)
    bits = K.relu_bits_like(6, 40, "cpu")
    f = K.gemm(a, b, act=K.ACT_RELU, relu_bits_out=bits)
    gy, w = torch.randn(6, 8, generator=g), torch.randn(40, 8, generator=g)
    assert torch.allclose(K.gemm(gy, w.t(), relu_bits=bits), K.gemm(gy, w.t(), relu_mask=f))
