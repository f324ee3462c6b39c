"""Layer kernels on the GPU against plain fp32 PyTorch references."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _C():
    from dlvk_b200 import _ext

    return _ext.C()


def close(a, b, tol):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    assert err <= tol * scale + 1e-6, f"max err {err}, scale {scale}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4, 1, 28, 28, 8, 3, 1, 1), (3, 8, 14, 14, 16, 3, 1, 1), (2, 3, 9, 11, 5, 3, 2, 0),
                                   (1300, 8, 14, 14, 16, 3, 1, 1)])  # more images than weight-gradient chunks
def test_conv2d(dtype, shape):
    # fp32 references without TF32 (cuDNN picks TF32 algorithms at large batch)
    with torch.backends.cudnn.flags(enabled=True, benchmark=False, deterministic=False, allow_tf32=False):
        _conv2d_case(dtype, shape)


def _conv2d_case(dtype, shape):
    C = _C()
    N, Cin, H, W, Cout, k, s, p = shape
    x = torch.randn(N, Cin, H, W, device="cuda")
    w = torch.randn(Cout, Cin, k, k, device="cuda") * 0.3
    b = torch.randn(Cout, device="cuda")
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    y = C.conv2d_fwd(x.to(dtype), w.to(dtype), b, s, p, True)
    ref = torch.relu(F.conv2d(x.to(dtype).float(), w.to(dtype).float(), b, stride=s, padding=p))
    close(y, ref, tol)
    g = torch.randn_like(ref)
    dx = C.conv2d_dgrad(g.to(dtype), w.to(dtype), list(x.shape), s, p, None)
    close(dx, torch.nn.grad.conv2d_input(list(x.shape), w.to(dtype).float(), g.to(dtype).float(), stride=s, padding=p), tol)
    dw = torch.zeros_like(w)
    db = torch.zeros(Cout, device="cuda")
    C.conv2d_wgrad(x.to(dtype), g.to(dtype), dw, db, s, p, False)
    close(dw, torch.nn.grad.conv2d_weight(x.to(dtype).float(), list(w.shape), g.to(dtype).float(), stride=s, padding=p), tol)
    close(db, g.to(dtype).float().sum((0, 2, 3)), tol)


def test_pooling():
    C = _C()
    x = torch.randn(3, 4, 10, 10, device="cuda")
    y, idx = C.maxpool_fwd(x, 2, 2)
    yr, ir = F.max_pool2d(x, 2, 2, return_indices=True)
    close(y, yr, 0)
    assert torch.equal(idx.long(), ir)
    g = torch.randn_like(y)
    xr = x.clone().requires_grad_(True)
    F.max_pool2d(xr, 2, 2).backward(g)
    close(C.maxpool_bwd(g, idx, 10, 10, 2, 2), xr.grad, 1e-6)
    # overlapping windows
    y, idx = C.maxpool_fwd(x, 3, 2)
    xr = x.clone().requires_grad_(True)
    F.max_pool2d(xr, 3, 2).backward(torch.ones_like(y))
    close(C.maxpool_bwd(torch.ones_like(y), idx, 10, 10, 3, 2), xr.grad, 1e-6)
    a = C.avgpool_fwd(x, 3, 2, 1)
    close(a, F.avg_pool2d(x, 3, 2, 1, count_include_pad=False), 1e-6)
    xr = x.clone().requires_grad_(True)
    F.avg_pool2d(xr, 3, 2, 1, count_include_pad=False).backward(torch.ones_like(a))
    close(C.avgpool_bwd(torch.ones_like(a), 10, 10, 3, 2, 1), xr.grad, 1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,p", [((256, 300), 0.1), ((64, 8, 5, 5), 0.0), ((1024, 4096), 0.1), ((24, 64), 0.1),
                                     ((16, 16, 14, 14), 0.1), ((7, 10, 3), 0.0)])
def test_batchnorm_relu_dropout(dtype, shape, p):
    """Covers the wide-grid reductions (several channel groups and row
    chunks), 8-wide element passes with channel wrap-around (S = 1 and S > 1)
    and the scalar fallbacks (C % 8 != 0, odd totals)."""
    from dlvk_b200.ops import nn as NN

    C = _C()
    torch.manual_seed(sum(shape))
    x = (torch.randn(*shape, device="cuda") * 2 + 1).to(dtype)
    Cn = shape[1]
    gamma = torch.rand(Cn, device="cuda") + 0.5
    beta = torch.randn(Cn, device="cuda") * 0.1
    rm, rv = torch.zeros(Cn, device="cuda"), torch.ones(Cn, device="cuda")
    y, mean, rstd = C.batchnorm_fwd(x, gamma, beta, rm, rv, 0.1, 1e-5, True, True, p, 3, 7, 5, None)
    rm_c, rv_c = torch.zeros(Cn), torch.ones(Cn)
    yr, mr, sr = NN.batchnorm_fwd(x.cpu(), gamma.cpu(), beta.cpu(), rm_c, rv_c, 0.1, 1e-5, True, True, p, 3, 7, 5)
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    close(y, yr, tol)
    close(rm, rm_c, 1e-4)
    close(rv, rv_c, 1e-4)
    ye, _, _ = C.batchnorm_fwd(x, gamma, beta, rm, rv, 0.1, 1e-5, False, True, p, 3, 7, 5, None)
    yer, _, _ = NN.batchnorm_fwd(x.cpu(), gamma.cpu(), beta.cpu(), rm_c, rv_c, 0.1, 1e-5, False, True, p, 3, 7, 5)
    close(ye, yer, tol)
    g = torch.randn(*shape, device="cuda").to(dtype)
    dg, dbt = torch.zeros(Cn, device="cuda"), torch.zeros(Cn, device="cuda")
    dx = C.batchnorm_bwd(x, g, mean, rstd, gamma, beta, dg, dbt, False, True, p, 3, 7, 5, None)
    dg_c, db_c = torch.zeros(Cn), torch.zeros(Cn)
    dxr = NN.batchnorm_bwd(x.cpu(), g.cpu(), mr, sr, gamma.cpu(), beta.cpu(), dg_c, db_c, False, True, p, 3, 7, 5)
    close(dx, dxr, tol * 2)
    close(dg, dg_c, tol * 2)
    close(dbt, db_c, tol * 2)
    # accumulate = True adds onto the existing parameter gradients
    C.batchnorm_bwd(x, g, mean, rstd, gamma, beta, dg, dbt, True, True, p, 3, 7, 5, None)
    close(dg, 2 * dg_c, tol * 2)
    close(dbt, 2 * db_c, tol * 2)


@pytest.mark.parametrize("rows", [333, 5003])  # 5003: more rows than one pass of the grid's warps covers
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [256, 512, 1024])  # bf16: one warp per row at 256, two warps per row at 512 / 1024
def test_layernorm(dtype, rows, D):
    C = _C()
    x = torch.randn(rows, D, device="cuda").to(dtype)
    gamma = torch.rand(D, device="cuda") + 0.5
    beta = torch.randn(D, device="cuda")
    y, mean, rstd = C.layernorm_fwd(x, gamma, beta, 1e-5)
    xr = x.float().clone().requires_grad_(True)
    gr = gamma.clone().requires_grad_(True)
    br = beta.clone().requires_grad_(True)
    yr = F.layer_norm(xr, (D,), gr, br, 1e-5)
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    close(y, yr, tol)
    g = torch.randn_like(yr).to(dtype)
    yr.backward(g.float())
    dgam, dbet = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    dx = C.layernorm_bwd(x, gamma, mean, rstd, g, dgam, dbet, False)
    close(dx, xr.grad, tol * 2)
    close(dgam, gr.grad, tol * 2)
    close(dbet, br.grad, tol * 2)
    dres = torch.randn_like(yr).to(dtype)
    cs = torch.full((D,), 2.0, device="cuda")
    dx2 = C.layernorm_bwd(x, gamma, mean, rstd, g, dgam, dbet, True, dres, dres_colsum=cs, dres_colsum_accumulate=True)
    close(dx2, xr.grad + dres.float(), tol * 2)
    close(dgam, 2 * gr.grad, tol * 2)
    close(cs, 2.0 + dres.float().sum(0), 1e-4)  # the residual gradient's column sums, fused


def test_dropout_matches_cpu_oracle():
    C = _C()
    n = 10001
    x = torch.ones(n, device="cuda")
    y = C.dropout(x, 0.25, 9, 1234, 3, None)
    keep = C.ref.dropout_mask(n, 0.25, 1234, 9, 3).bool()
    assert torch.equal((y.cpu() != 0), keep)
    assert abs(keep.float().mean().item() - 0.75) < 0.02
    close(y.cpu()[keep], torch.full((int(keep.sum()),), 1 / 0.75), 1e-6)
    st = torch.tensor([3], dtype=torch.int64, device="cuda")
    y2 = C.dropout(x, 0.25, 9, 1234, 0, st)
    assert torch.equal(y, y2)


def test_embedding():
    C = _C()
    table = torch.randn(100, 64, device="cuda")
    ids = torch.tensor([[0, 5, 99], [100, -1, 5]], dtype=torch.int32, device="cuda")
    out = C.embedding_fwd(ids, table)
    ref = table[ids.clamp(0, 99).long()]
    ref[1, 0] = 0
    ref[1, 1] = 0
    close(out, ref, 0)
    g = torch.randn(2, 3, 64, device="cuda")
    dt = torch.zeros(100, 64, device="cuda")
    C.embedding_bwd(ids, g, dt)
    ref = torch.zeros(100, 64, device="cuda")
    ref[0] += g[0, 0]
    ref[5] += g[0, 1] + g[1, 2]
    ref[99] += g[0, 2]
    close(dt, ref, 1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention(dtype):
    from dlvk_b200.ops import nn as NN

    B, S, H, D = 2, 128, 4, 64
    E = H * D
    qkv = torch.randn(B, S, 3 * E, device="cuda").to(dtype)
    scale = 1 / math.sqrt(D)
    out, probs = NN.attention_fwd(qkv, B, S, H, D, scale)
    x = qkv.float().reshape(B, S, 3, H, D).clone().requires_grad_(True)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    ref = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B, S, E)
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    close(out, ref, tol)
    g = torch.randn(B, S, E, device="cuda")
    ref.backward(g)
    dqkv = NN.attention_bwd(qkv, probs, g.to(dtype), B, S, H, D, scale, out=out)
    close(dqkv, x.grad.reshape(B, S, 3 * E), tol * 3)
