"""Fused tcgen05 attention (forward and backward) against an fp32 PyTorch
reference of the same op on the same bf16 inputs."""
import math

import pytest
import torch

from dlvk_b200 import _ext

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def ref_attention(qkv, B, S, H, D, scale):
    x = qkv.float().reshape(B, S, 3, H, D).requires_grad_(True)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    p = torch.softmax(s, -1)
    o = torch.matmul(p, v).transpose(1, 2).reshape(B, S, H * D)
    lse2 = torch.logsumexp(s, -1) / math.log(2.0)  # [B, H, S] in log2 units
    return x, o, lse2


def _check_err():
    C = _ext.C()
    torch.cuda.synchronize()
    assert C.read_device_error() == 0


@pytest.mark.parametrize("B,S,H", [(1, 128, 1), (2, 256, 2), (3, 512, 4), (16, 512, 16), (2, 1024, 3)])
@pytest.mark.parametrize("max_ctas", [0, 3])
def test_flash_forward_backward(B, S, H, max_ctas):
    D = 64
    scale = 1.0 / math.sqrt(D)
    g = torch.Generator().manual_seed(B * 1000 + S + H)
    qkv = (torch.randn(B, S, 3 * H * D, generator=g) * 1.5).to(DEV, torch.bfloat16)
    C = _ext.C()
    assert C.flash_attn_supported(B, S, H, D, qkv)
    out, lse = C.flash_attn_fwd(qkv, B, S, H, scale, max_ctas)
    _check_err()
    x, o_ref, lse_ref = ref_attention(qkv, B, S, H, D, scale)
    assert torch.allclose(lse, lse_ref.detach(), atol=2e-3, rtol=1e-4)
    err = (out.float() - o_ref.detach()).abs().max().item()
    assert err < 2e-2 * max(1.0, o_ref.abs().max().item()), err
    dout = (torch.randn(B, S, H * D, generator=g)).to(DEV, torch.bfloat16)
    o_ref.backward(dout.float())
    dref = x.grad.reshape(B, S, 3 * H * D)
    dqkv = C.flash_attn_bwd(qkv, out, dout, lse, B, S, H, scale, max_ctas)
    _check_err()
    for part, name in ((0, "dq"), (1, "dk"), (2, "dv")):
        a = dqkv.float().reshape(B, S, 3, H * D)[:, :, part]
        r = dref.reshape(B, S, 3, H * D)[:, :, part]
        rel = ((a - r).norm() / r.norm()).item()
        assert rel < 2.5e-2, (name, rel)


def test_attention_layer_uses_fused_path():
    """A bf16 MultiHeadAttention layer with S % 128 == 0 runs the fused
    kernels and matches the GEMM + softmax path."""
    import os

    from dlvk_b200.models import layers as L

    torch.manual_seed(0)
    lay = L.MultiHeadAttentionLayer(256, 4)
    twin = lay.clone()
    lay.to(DEV, torch.bfloat16)
    twin.to(DEV, torch.bfloat16)
    x = torch.randn(4, 256, 256, device=DEV).bfloat16()
    g = torch.randn(4, 256, 256, device=DEV).bfloat16()
    y1 = lay.forward(x)
    dx1 = lay.backward(g)
    os.environ["DLVK_FLASH_ATTN"] = "0"
    try:
        y0 = twin.forward(x)
        dx0 = twin.backward(g)
    finally:
        os.environ.pop("DLVK_FLASH_ATTN")
    assert ((y1.float() - y0.float()).norm() / y0.float().norm()).item() < 2e-2
    assert ((dx1.float() - dx0.float()).norm() / dx0.float().norm()).item() < 3e-2
    for a, b in zip(lay.parameters(), twin.parameters()):
        assert ((a.grad - b.grad).norm() / b.grad.norm()).item() < 3e-2, a.name


@pytest.mark.multigpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two CUDA devices")
def test_kernels_on_two_devices_in_one_process():
    """One process driving two GPUs: the kernels whose launchers raise the
    dynamic shared-memory limit (fused attention, the persistent softmax-CE,
    the tensor-core GEMM) must do so on each device before launching there."""
    C = _ext.C()
    B, S, H, D = 2, 256, 2, 64
    scale = 1.0 / math.sqrt(D)
    for dev in ("cuda:0", "cuda:1"):
        with torch.cuda.device(dev):
            g = torch.Generator().manual_seed(7)
            qkv = torch.randn(B, S, 3 * H * D, generator=g).to(dev, torch.bfloat16)
            out, lse = C.flash_attn_fwd(qkv, B, S, H, scale, 0)
            x, o_ref, lse_ref = ref_attention(qkv.to("cuda:0"), B, S, H, D, scale)
            err = (out.float().to("cuda:0") - o_ref.detach()).abs().max().item()
            assert err < 2e-2 * max(1.0, o_ref.abs().max().item()), (dev, err)
            dqkv = C.flash_attn_bwd(qkv, out, torch.ones_like(out), lse, B, S, H, scale, 0)
            assert torch.isfinite(dqkv.float()).all()
            logits = torch.randn(300, 32000, generator=g).to(dev, torch.bfloat16)
            lab = torch.randint(0, 32000, (300,), generator=g, dtype=torch.int32).to(dev)
            loss_rows, _ = C.softmax_ce(logits, lab, 1.0)
            ref = torch.nn.functional.cross_entropy(logits.float(), lab.long(), reduction="none")
            torch.testing.assert_close(loss_rows, ref, atol=0.05, rtol=1e-2)
            a = torch.randn(512, 256, generator=g).to(dev, torch.bfloat16)
            b = torch.randn(256, 1024, generator=g).to(dev, torch.bfloat16)
            c = C.gemm(a, b, force_path=1)
            assert (c.float() - a.float() @ b.float()).abs().max().item() < 2e-2 * (a.float() @ b.float()).abs().max().item()
            torch.cuda.synchronize(dev)
            # the error word is per device: read this device's, with it current
            assert C.read_device_error(True) == 0, dev
