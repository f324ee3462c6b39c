"""Implicit-GEMM tcgen05 convolution (conv_tc.cu) against plain fp32 PyTorch
convolutions of the same bf16-rounded operands."""
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


@pytest.fixture
def tc_mode():
    C = _C()
    old = C.conv_tc_get_mode()
    C.conv_tc_set_mode(1)
    yield C
    C.conv_tc_set_mode(old)


# (N, Cin, H, W, Cout, k, stride, pad): 64/128/256-wide column tiles, ragged
# pixel counts, strided and 1x1 filters, padding larger than one.  The last
# two are 1x1 convolutions whose pixel counts are multiples of 8: they run as
# batched GEMMs over the NCHW tensors (ragged row tiles: 272 and 32 channels).
SHAPES = [(4, 16, 12, 12, 32, 3, 1, 1), (2, 64, 17, 17, 128, 3, 2, 1), (2, 24, 9, 9, 200, 5, 1, 2),
          (3, 128, 10, 7, 64, 1, 1, 0), (2, 32, 15, 15, 48, 3, 2, 0), (1, 16, 8, 8, 16, 7, 1, 3),
          (2, 64, 8, 12, 96, 1, 1, 0), (3, 32, 16, 16, 272, 1, 1, 0)]


@pytest.mark.parametrize("shape", SHAPES)
def test_conv_tc_forward(tc_mode, shape):
    C = tc_mode
    N, Cin, H, W, Cout, k, s, p = shape
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(N, Cin, H, W, device="cuda", generator=g).bfloat16()
    w = (torch.randn(Cout, Cin, k, k, device="cuda", generator=g) * 0.2).bfloat16()
    b = torch.randn(Cout, device="cuda", generator=g)
    for relu in (False, True):
        y = C.conv2d_fwd(x, w, b, s, p, relu)
        ref = F.conv2d(x.float(), w.float(), b, stride=s, padding=p)
        if relu:
            ref = torch.relu(ref)
        assert y.dtype == torch.bfloat16 and y.shape == ref.shape
        close(y, ref, 1e-2)


@pytest.mark.parametrize("shape", SHAPES)
def test_conv_tc_dgrad(tc_mode, shape):
    C = tc_mode
    N, Cin, H, W, Cout, k, s, p = shape
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(Cout, Cin, k, k, device="cuda", generator=g) * 0.2).bfloat16()
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    gy = torch.randn(N, Cout, Ho, Wo, device="cuda", generator=g).bfloat16()
    ref = torch.nn.grad.conv2d_input([N, Cin, H, W], w.float(), gy.float(), stride=s, padding=p)
    dx = C.conv2d_dgrad(gy, w, [N, Cin, H, W], s, p, None)
    close(dx, ref, 1e-2)
    mask = torch.randn(N, Cin, H, W, device="cuda", generator=g).bfloat16()
    dxm = C.conv2d_dgrad(gy, w, [N, Cin, H, W], s, p, mask)
    close(dxm, torch.where(mask.float() > 0, ref, torch.zeros_like(ref)), 1e-2)


@pytest.mark.parametrize("shape", SHAPES)
def test_conv_tc_wgrad(tc_mode, shape):
    C = tc_mode
    N, Cin, H, W, Cout, k, s, p = shape
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(N, Cin, H, W, device="cuda", generator=g).bfloat16()
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    gy = torch.randn(N, Cout, Ho, Wo, device="cuda", generator=g).bfloat16()
    ref = torch.nn.grad.conv2d_weight(x.float(), [Cout, Cin, k, k], gy.float(), stride=s, padding=p)
    dw = torch.zeros(Cout, Cin, k, k, device="cuda")
    db = torch.zeros(Cout, device="cuda")
    C.conv2d_wgrad(x, gy, dw, db, s, p, False)
    close(dw, ref, 1e-2)
    close(db, gy.float().sum((0, 2, 3)), 1e-3)
    C.conv2d_wgrad(x, gy, dw, db, s, p, True)  # accumulate
    close(dw, 2 * ref, 1e-2)


def test_conv_tc_large_wgrad_split(tc_mode):
    """Many pixel blocks: the reduction is split across CTAs."""
    C = tc_mode
    N, Cin, H, W, Cout = 8, 64, 32, 32, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(N, Cin, H, W, device="cuda", generator=g).bfloat16()
    gy = torch.randn(N, Cout, H, W, device="cuda", generator=g).bfloat16()
    ref = torch.nn.grad.conv2d_weight(x.float(), [Cout, Cin, 3, 3], gy.float(), stride=1, padding=1)
    dw = torch.zeros(Cout, Cin, 3, 3, device="cuda")
    C.conv2d_wgrad(x, gy, dw, None, 1, 1, False)
    close(dw, ref, 1e-2)
    assert int(C.read_device_error(True)) == 0


def test_conv_tc_layer_training():
    """A bf16 CNN with 32/64-channel convolutions trains through the layer API
    on the automatic path (the second convolution is large enough to take the
    tensor-core implicit GEMM) and matches the direct kernels."""
    import dlvk_b200 as dl
    from dlvk_b200.models.sequential import Sequential
    from dlvk_b200.training.step import TrainStep

    C = _C()
    x = torch.rand(64, 16, 32, 32, generator=torch.Generator().manual_seed(0))
    y = torch.randint(0, 10, (64,), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    losses = {}
    old = C.conv_tc_get_mode()
    try:
        for mode in (1, 2):
            C.conv_tc_set_mode(mode)
            m = Sequential("cuda:0", "bf16", seed=0)
            m.add_conv2d(16, 64, 3, 1, 1).add_relu().add_maxpool2d(2, 2)
            m.add_conv2d(64, 64, 3, 1, 1).add_relu().add_maxpool2d(2, 2)
            m.add_flatten().add_dense(64 * 8 * 8, 10).add_softmax()
            m.build()
            step = TrainStep(m, dl.CrossEntropyLoss(), dl.Adam(1e-3), graph=False)
            ls = [float(step(x, y).detach()) for _ in range(5)]
            step.close()
            losses[mode] = ls
    finally:
        C.conv_tc_set_mode(old)
    assert losses[1][-1] < losses[1][0]
    for a, b in zip(losses[1], losses[2]):
        assert abs(a - b) <= 0.05 * abs(b) + 1e-3, losses
