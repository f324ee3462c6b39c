"""The reference's full TensorOps instance API (include/dlvk/tensor/
tensor_ops.h:28-120) against plain fp32 PyTorch, on CPU and on the GPU."""
import pytest
import torch
import torch.nn.functional as F

from dlvk_b200.tensor import Tensor, TensorOps

DEVICES = ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)]


def T(x):
    return Tensor.wrap(x.contiguous())


def empty_like(x):
    return Tensor.wrap(torch.empty_like(x))


@pytest.mark.parametrize("dev", DEVICES)
def test_elementwise_scalar_and_batched(dev):
    ops = TensorOps(dev if dev == "cpu" else "cuda:0")
    g = torch.Generator().manual_seed(0)
    a = torch.randn(3, 5, 7, generator=g).to(dev)
    b = torch.randn(3, 7, 4, generator=g).to(dev)
    r = Tensor.wrap(torch.empty(3, 5, 4, device=dev))
    assert ops.batch_matrix_multiply(T(a), T(b), r)
    torch.testing.assert_close(r.data, torch.bmm(a, b), rtol=1e-2, atol=1e-2)
    x = torch.rand(64, generator=g).to(dev) + 0.1
    y = torch.randn(64, generator=g).to(dev)
    out = empty_like(x)
    assert ops.element_wise_multiply(T(x), T(y), out)
    torch.testing.assert_close(out.data, x * y)
    assert ops.element_wise_sqrt(T(x), out)
    torch.testing.assert_close(out.data, x.sqrt())
    assert ops.element_wise_square(T(y), out)
    torch.testing.assert_close(out.data, y * y)
    assert ops.scale(T(y), 2.5, out)
    torch.testing.assert_close(out.data, y * 2.5)
    assert ops.scalar_add(T(y), -1.25, out)
    torch.testing.assert_close(out.data, y - 1.25)
    assert ops.validate_element_wise_operation(T(x), T(y), out)
    assert not ops.validate_matrix_multiply(T(x), T(y), out)


@pytest.mark.parametrize("dev", DEVICES)
def test_adam_update_and_clipping(dev):
    ops = TensorOps(dev if dev == "cpu" else "cuda:0")
    g = torch.Generator().manual_seed(1)
    p = torch.randn(256, generator=g).to(dev)
    grad = torch.randn(256, generator=g).to(dev)
    m = torch.randn(256, generator=g).to(dev) * 0.1
    v = torch.rand(256, generator=g).to(dev) * 0.1
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    mr = 0.9 * mr + 0.1 * grad
    vr = 0.999 * vr + 0.001 * grad * grad
    pr = pr - 1e-2 * mr / (vr.sqrt() + 1e-8)  # bias corrections of 1, as the reference's GPU path
    P, M, V = T(p), T(m), T(v)
    nm, nv = empty_like(m), empty_like(v)
    assert ops.adam_update(T(grad), M, V, P, nm, nv, 1e-2, 0.9, 0.999, 1e-8)
    torch.testing.assert_close(P.data, pr, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(nm.data, mr, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(nv.data, vr, rtol=1e-5, atol=1e-6)
    out = empty_like(grad)
    norm = float(grad.norm())
    assert ops.gradient_clip_by_norm(T(grad), norm / 2, out)
    torch.testing.assert_close(out.data, grad * 0.5, rtol=1e-4, atol=1e-5)
    assert ops.gradient_clip_by_norm(T(grad), norm * 2, out)
    torch.testing.assert_close(out.data, grad)
    assert ops.gradient_clip_by_value(T(grad), -0.5, 0.5, out)
    torch.testing.assert_close(out.data, grad.clamp(-0.5, 0.5))


@pytest.mark.parametrize("dev", DEVICES)
def test_conv_pool_bn_dropout(dev):
    ops = TensorOps(dev if dev == "cpu" else "cuda:0")
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 3, 8, 8, generator=g).to(dev)
    w = torch.randn(4, 3, 3, 3, generator=g).to(dev) * 0.3
    b = torch.randn(4, generator=g).to(dev)
    y = Tensor.wrap(torch.empty(2, 4, 8, 8, device=dev))
    assert ops.conv2d(T(x), T(w), T(b), y, 1, 1, 1, 1)
    torch.testing.assert_close(y.data, F.conv2d(x, w, b, padding=1), rtol=1e-4, atol=1e-4)
    gy = torch.randn(2, 4, 8, 8, generator=g).to(dev)
    dx = Tensor.wrap(torch.empty_like(x))
    assert ops.conv2d_backward_input(T(gy), T(w), dx, 1, 1, 1, 1)
    torch.testing.assert_close(dx.data, torch.nn.grad.conv2d_input(list(x.shape), w, gy, padding=1), rtol=1e-4,
                               atol=1e-4)
    dw, db = Tensor.wrap(torch.empty_like(w)), Tensor.wrap(torch.empty_like(b))
    assert ops.conv2d_backward_weight(T(x), T(gy), dw, db, 1, 1, 1, 1)
    torch.testing.assert_close(dw.data, torch.nn.grad.conv2d_weight(x, list(w.shape), gy, padding=1), rtol=1e-4,
                               atol=1e-3)
    torch.testing.assert_close(db.data, gy.sum((0, 2, 3)), rtol=1e-4, atol=1e-4)
    # pooling
    mp = Tensor.wrap(torch.empty(2, 3, 4, 4, device=dev))
    idx = Tensor.wrap(torch.empty(2, 3, 4, 4, dtype=torch.int32, device=dev))
    assert ops.maxpool2d(T(x), mp, idx, 2, 2, 2, 2, 0, 0)
    torch.testing.assert_close(mp.data, F.max_pool2d(x, 2))
    gp = torch.randn(2, 3, 4, 4, generator=g).to(dev)
    gi = Tensor.wrap(torch.empty_like(x))
    assert ops.maxpool2d_backward(T(gp), idx, gi)
    xr = x.clone().requires_grad_(True)
    F.max_pool2d(xr, 2).backward(gp)
    torch.testing.assert_close(gi.data, xr.grad)
    ap = Tensor.wrap(torch.empty(2, 3, 4, 4, device=dev))
    assert ops.avgpool2d(T(x), ap, 2, 2, 2, 2, 0, 0)
    torch.testing.assert_close(ap.data, F.avg_pool2d(x, 2))
    assert ops.avgpool2d_backward(T(gp), gi, 2, 2, 2, 2, 0, 0)
    xr = x.clone().requires_grad_(True)
    F.avg_pool2d(xr, 2).backward(gp)
    torch.testing.assert_close(gi.data, xr.grad)
    # batch norm
    gamma, beta = torch.rand(3, generator=g).to(dev) + 0.5, torch.randn(3, generator=g).to(dev)
    rm, rv = torch.zeros(3, device=dev), torch.ones(3, device=dev)
    out, sm, sv = Tensor.wrap(torch.empty_like(x)), Tensor.wrap(torch.empty(3, device=dev)), \
        Tensor.wrap(torch.empty(3, device=dev))
    assert ops.batch_norm(T(x), T(gamma), T(beta), Tensor.wrap(rm), Tensor.wrap(rv), out, sm, sv, 0.1, 1e-5, True)
    ref = F.batch_norm(x, None, None, gamma, beta, True, 0.1, 1e-5)
    torch.testing.assert_close(out.data, ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(sv.data, x.var((0, 2, 3), unbiased=False), rtol=1e-3, atol=1e-4)
    gx, gg, gb = Tensor.wrap(torch.empty_like(x)), Tensor.wrap(torch.empty(3, device=dev)), \
        Tensor.wrap(torch.empty(3, device=dev))
    go = torch.randn_like(x)
    assert ops.batch_norm_backward(T(go), T(x), T(gamma), sm, sv, gx, gg, gb, 1e-5)
    xr, gr, br = x.clone().requires_grad_(True), gamma.clone().requires_grad_(True), beta.clone().requires_grad_(True)
    F.batch_norm(xr, None, None, gr, br, True, 0.1, 1e-5).backward(go)
    torch.testing.assert_close(gx.data, xr.grad, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gg.data, gr.grad, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gb.data, br.grad, rtol=1e-3, atol=1e-3)
    # dropout: mask in {0,1}, kept values scaled by 1/(1-p); backward uses the mask
    z = torch.randn(4096, generator=g).to(dev)
    o, mk = Tensor.wrap(torch.empty_like(z)), Tensor.wrap(torch.empty_like(z))
    assert ops.dropout(T(z), o, mk, 0.25, True, 7)
    keep = mk.data != 0
    assert 0.65 < float(keep.float().mean()) < 0.85
    torch.testing.assert_close(o.data[keep], z[keep] / 0.75)
    assert float(o.data[~keep].abs().max()) == 0.0
    gz = Tensor.wrap(torch.empty_like(z))
    assert ops.dropout_backward(T(torch.ones_like(z)), mk, gz, 0.25)
    torch.testing.assert_close(gz.data, keep.float() / 0.75)
    assert ops.dropout(T(z), o, mk, 0.25, False, 7)
    torch.testing.assert_close(o.data, z)


@pytest.mark.parametrize("dev", DEVICES)
def test_embedding_layernorm_attention_reshapes(dev):
    ops = TensorOps(dev if dev == "cpu" else "cuda:0")
    g = torch.Generator().manual_seed(3)
    table = torch.randn(50, 16, generator=g).to(dev)
    ids = torch.randint(0, 50, (4, 6), generator=g).to(dev)
    out = Tensor.wrap(torch.empty(4, 6, 16, device=dev))
    assert ops.embedding_lookup(out, T(ids), T(table))
    torch.testing.assert_close(out.data, table[ids])
    x = torch.randn(12, 64, generator=g).to(dev)
    w, b = torch.rand(64, generator=g).to(dev) + 0.5, torch.randn(64, generator=g).to(dev)
    y = empty_like(x)
    assert ops.layer_norm(y, T(x), T(w), T(b), 1e-5)
    torch.testing.assert_close(y.data, F.layer_norm(x, (64,), w, b, 1e-5), rtol=1e-4, atol=1e-4)
    B, S, H, D = 2, 5, 3, 4
    inp = torch.randn(B, S, H * D, generator=g).to(dev)
    heads = Tensor.wrap(torch.empty(B, H, S, D, device=dev))
    assert ops.reshape_for_attention(heads, T(inp), B, S, H, D)
    torch.testing.assert_close(heads.data, inp.reshape(B, S, H, D).permute(0, 2, 1, 3))
    back = Tensor.wrap(torch.empty(B, S, H * D, device=dev))
    assert ops.reshape_from_attention(back, heads, B, S, H, D)
    torch.testing.assert_close(back.data, inp)
    q, k, v = (torch.randn(B * H, S, D, generator=g).to(dev) for _ in range(3))
    att = Tensor.wrap(torch.empty(B * H, S, D, device=dev))
    assert ops.attention(att, T(q), T(k), T(v), 0.5)
    ref = torch.softmax(q @ k.transpose(-1, -2) * 0.5, -1) @ v
    torch.testing.assert_close(att.data, ref, rtol=2e-2, atol=2e-2)
    TensorOps.shutdown()
