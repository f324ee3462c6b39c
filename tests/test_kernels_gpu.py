"""Elementwise, reduction, softmax/loss and optimizer kernels against plain
fp32 PyTorch references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from dlvk_b200 import _ext

    return _ext.C()


UN = dict(relu=0, sigmoid=1, tanh=2, scale=3, clamp=4, sqrt=5, copy=6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unary_binary(dtype):
    C = _C()
    x = torch.randn(1000003, device="cuda").to(dtype)
    y = torch.randn(1000003, device="cuda").to(dtype)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(C.unary(x, UN["relu"]).float(), torch.relu(x.float()), atol=tol, rtol=tol)
    torch.testing.assert_close(C.unary(x, UN["sigmoid"]).float(), torch.sigmoid(x.float()), atol=tol * 2, rtol=tol * 2)
    torch.testing.assert_close(C.unary(x, UN["tanh"]).float(), torch.tanh(x.float()), atol=tol * 2, rtol=tol * 2)
    torch.testing.assert_close(C.unary(x, UN["clamp"], -0.5, 0.5).float(), x.float().clamp(-0.5, 0.5))
    torch.testing.assert_close(C.binary(x, y, 0).float(), (x.float() + y.float()).to(dtype).float(), atol=tol, rtol=tol)
    torch.testing.assert_close(C.binary(x, y, 2).float(), (x.float() * y.float()).to(dtype).float(), atol=tol, rtol=tol)
    # guarded divide: |b| < 1e-8 -> sign(a) * 1e8
    a = torch.tensor([1.0, -2.0, 3.0], device="cuda")
    b = torch.tensor([0.0, 0.0, 2.0], device="cuda")
    torch.testing.assert_close(C.binary(a, b, 3), torch.tensor([1e8, -1e8, 1.5], device="cuda"))


def test_reductions():
    C = _C()
    x = torch.randn(3001, 517, device="cuda")
    torch.testing.assert_close(C.reduce(x, 0).cpu(), x.sum().cpu(), rtol=1e-4, atol=1e-2)
    torch.testing.assert_close(C.reduce(x, 1).cpu(), x.max().cpu())
    torch.testing.assert_close(C.reduce(x, 2).cpu(), x.min().cpu())
    torch.testing.assert_close(C.colsum(x), x.sum(0), rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(C.rowsum(x), x.sum(1), rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(C.transpose(x), x.t().contiguous())
    y = torch.randn(2, 3, 4, 5, device="cuda")
    torch.testing.assert_close(C.permute4(y, [0, 2, 1, 3]), y.permute(0, 2, 1, 3).contiguous())


@pytest.mark.parametrize("cols", [10, 47, 1000, 32000])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_softmax_ce(cols, dtype):
    C = _C()
    rows = 37
    x = (torch.randn(rows, cols, device="cuda") * 3).to(dtype)
    lab = torch.randint(0, cols, (rows,), device="cuda", dtype=torch.int32)
    loss_rows, dl = C.softmax_ce(x, lab, 1.0 / rows)
    xf = x.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(xf, lab.long(), reduction="none")
    ref.mean().backward()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(loss_rows, ref.detach(), atol=tol * 10, rtol=tol)
    torch.testing.assert_close(dl.float(), xf.grad, atol=tol, rtol=tol * 10)
    sm = C.softmax(x)
    torch.testing.assert_close(sm.float(), torch.softmax(x.float(), -1), atol=tol, rtol=tol * 10)


@pytest.mark.parametrize("cols", [8000, 32000])
@pytest.mark.parametrize("rows", [19, 700])
def test_softmax_ce_vocab_inplace_ignored(cols, rows):
    """bf16 vocabulary-sized rows (register-resident kernels; with 700 rows
    each persistent block walks several rows and prefetches the next),
    gradient written over the logits, one ignored row."""
    C = _C()
    x = (torch.randn(rows, cols, device="cuda") * 3).bfloat16()
    lab = torch.randint(0, cols, (rows,), device="cuda", dtype=torch.int32)
    lab[3] = -1
    xf = x.float().requires_grad_(True)
    keep = lab >= 0
    ref = torch.nn.functional.cross_entropy(xf, lab.long().clamp(min=0), reduction="none") * keep
    ref.sum().backward()
    loss_rows, dl = C.softmax_ce(x, lab, 1.0, in_place=True)
    assert dl.data_ptr() == x.data_ptr()
    torch.testing.assert_close(loss_rows, ref.detach(), atol=0.2, rtol=2e-2)
    torch.testing.assert_close(dl.float(), xf.grad, atol=2e-2, rtol=0.2)
    assert float(dl[3].float().abs().max()) == 0.0


def test_softmax_bwd_and_losses():
    C = _C()
    x = torch.randn(64, 100, device="cuda", requires_grad=True)
    y = torch.softmax(x, -1)
    dy = torch.randn_like(y)
    y.backward(dy)
    dx = C.softmax_bwd(y.detach(), dy)
    torch.testing.assert_close(dx, x.grad, atol=1e-5, rtol=1e-4)
    p = torch.rand(1000, device="cuda") * 0.98 + 0.01
    t = (torch.rand(1000, device="cuda") > 0.5).float()
    l, g = C.pointwise_loss(p, t, 0, 1.0 / 1000, 1.0 / 1000, True)
    torch.testing.assert_close(l, ((p - t) ** 2).mean(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(g, 2 * (p - t) / 1000)
    l, g = C.pointwise_loss(p, t, 1, 1.0 / 1000, 1.0 / 1000, True)
    torch.testing.assert_close(l, torch.nn.functional.binary_cross_entropy(p, t), rtol=1e-5, atol=1e-6)


def _hyper(lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, mom=0.0, alpha=0.99, gs=1.0):
    from dlvk_b200.ops.optim_kernels import make_hyper

    return make_hyper(torch.device("cuda"), lr=lr, beta1=b1, beta2=b2, eps=eps, weight_decay=wd, momentum=mom,
                      alpha=alpha, grad_scale=gs)


def test_adam_matches_reference():
    C = _C()
    n = 100003
    p = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    h = _hyper()
    for step in range(1, 4):
        g = torch.randn(n, device="cuda")
        C.optim_advance(h)
        C.optim_update(1, h, p, g, m, v)
        mr = 0.9 * mr + 0.1 * g
        vr = 0.999 * vr + 0.001 * g * g
        mh = mr / (1 - 0.9 ** step)
        vh = vr / (1 - 0.999 ** step)
        pr = pr - 1e-3 * mh / (vh.sqrt() + 1e-8)
    torch.testing.assert_close(p, pr, atol=1e-6, rtol=1e-5)


def test_sgd_momentum_and_rmsprop():
    C = _C()
    n = 5000
    p = torch.randn(n, device="cuda")
    buf = torch.zeros(n, device="cuda")
    pr, br = p.clone(), buf.clone()
    h = _hyper(lr=0.1, mom=0.9)
    for _ in range(3):
        g = torch.randn(n, device="cuda")
        C.optim_advance(h)
        C.optim_update(0, h, p, g, buf, None)
        br = 0.9 * br + g
        pr = pr - 0.1 * br
    torch.testing.assert_close(p, pr, atol=1e-6, rtol=1e-5)
    p = torch.randn(n, device="cuda")
    sq = torch.zeros(n, device="cuda")
    pr, sr = p.clone(), sq.clone()
    h = _hyper(lr=0.01, alpha=0.99, eps=1e-8)
    for _ in range(3):
        g = torch.randn(n, device="cuda")
        C.optim_advance(h)
        C.optim_update(2, h, p, g, None, sq)
        sr = 0.99 * sr + 0.01 * g * g
        pr = pr - 0.01 * g / (sr.sqrt() + 1e-8)
    torch.testing.assert_close(p, pr, atol=1e-6, rtol=1e-5)


def test_grad_stats_and_clip():
    C = _C()
    g = torch.randn(77777, device="cuda")
    sumsq = torch.zeros(1, device="cuda")
    flag = torch.zeros(1, device="cuda", dtype=torch.int32)
    clip = torch.zeros(1, device="cuda")
    scratch = torch.empty(C.grad_stats_scratch_floats(), device="cuda")
    C.grad_stats(g, 1.0, 1.0, sumsq, flag, clip, False, scratch)
    norm = g.norm().item()
    assert math.isclose(sumsq.item(), norm * norm, rel_tol=1e-4)
    assert flag.item() == 0
    assert math.isclose(clip.item(), min(1.0, 1.0 / (norm + 1e-6)), rel_tol=1e-4)
    g[5] = float("inf")
    C.grad_stats(g, 1.0, 0.0, sumsq, flag, None, False, scratch)
    assert flag.item() == 1


def test_softmax_ce_vocab_confident_label_gradient():
    """Rows whose label dominates (p close to 1): the label's gradient p - 1 is
    small and must stay accurate, so it is computed in fp32 from the logit and
    not from the bf16-rounded probability."""
    C = _C()
    rows, cols = 300, 32000
    x = torch.randn(rows, cols, device="cuda")
    lab = torch.randint(0, cols, (rows,), device="cuda", dtype=torch.int32)
    x[torch.arange(rows), lab.long()] += 20.0
    x = x.bfloat16()
    xf = x.float().requires_grad_(True)
    torch.nn.functional.cross_entropy(xf, lab.long(), reduction="sum").backward()
    _, dl = C.softmax_ce(x, lab, 1.0, in_place=False)
    ref_l = xf.grad[torch.arange(rows), lab.long()]
    got_l = dl.float()[torch.arange(rows), lab.long()]
    # p - 1 is about -1e-4 here: rounding p to bf16 first would give 0
    assert float(ref_l.abs().max()) < 1e-2
    torch.testing.assert_close(got_l, ref_l, atol=1e-6, rtol=2e-2)
    torch.testing.assert_close(dl.float(), xf.grad, atol=1e-3, rtol=2e-2)
