"""Attention micro-benchmark: the fused tcgen05 kernels against the
GEMM + softmax path and against PyTorch's scaled_dot_product_attention
(cuDNN and flash backends, same bf16 inputs and layout), forward and
backward, CUDA-event timed with L2 flushed between iterations.

    python -m dlvk_b200.bench.attention [--B 16 --S 512 --H 16] [--iters 20]
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from dlvk_b200.bench.common import measured_peaks, time_fn
from dlvk_b200.ops import nn as NN


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--S", type=int, default=512)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    B, S, H, D = a.B, a.S, a.H, 64
    scale = 1.0 / math.sqrt(D)
    qkv = torch.randn(B, S, 3 * H * D, device="cuda").bfloat16()
    dout = torch.randn(B, S, H * D, device="cuda").bfloat16()
    flops_f = 4.0 * B * H * S * S * D
    peak = measured_peaks()["bf16_tflops"]
    res = {"B": B, "S": S, "H": H, "D": D}
    for mode in ("fused", "unfused"):
        if mode == "unfused":
            os.environ["DLVK_FLASH_ATTN"] = "0"
        out, aux = NN.attention_fwd(qkv, B, S, H, D, scale)
        tf = time_fn(lambda: NN.attention_fwd(qkv, B, S, H, D, scale), a.iters)
        tb = time_fn(lambda: NN.attention_bwd(qkv, aux, dout, B, S, H, D, scale, out=out), a.iters)
        res[mode] = {"fwd_ms": round(tf, 4), "bwd_ms": round(tb, 4),
                     "fwd_tflops": round(flops_f / tf / 1e9, 1), "bwd_tflops": round(2.5 * flops_f / tb / 1e9, 1),
                     "fwd_frac_of_measured": round(flops_f / tf / 1e9 / peak, 3)}
    os.environ.pop("DLVK_FLASH_ATTN", None)
    res["speedup_fwd"] = round(res["unfused"]["fwd_ms"] / res["fused"]["fwd_ms"], 2)
    res["speedup_bwd"] = round(res["unfused"]["bwd_ms"] / res["fused"]["bwd_ms"], 2)
    # PyTorch SDPA on the same [B, S, 3, H, D] buffer (strided [B, H, S, D] views).
    from torch.nn.attention import SDPBackend, sdpa_kernel

    v5 = qkv.view(B, S, 3, H, D)
    q, k, v = (v5[:, :, i].transpose(1, 2).detach().requires_grad_(True) for i in range(3))
    go = dout.view(B, S, H, D).transpose(1, 2)
    for name, be in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                o = torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale)
                tf = time_fn(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale), a.iters)
                tfb = time_fn(lambda: torch.autograd.grad(
                    torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=scale), (q, k, v), go), a.iters)
            tb = max(tfb - tf, 1e-6)
            res[name] = {"fwd_ms": round(tf, 4), "bwd_ms": round(tb, 4), "fwd_tflops": round(flops_f / tf / 1e9, 1),
                         "bwd_tflops": round(2.5 * flops_f / tb / 1e9, 1)}
            res["ours_vs_" + name] = {"fwd": round(tf / res["fused"]["fwd_ms"], 3),
                                      "bwd": round(tb / res["fused"]["bwd_ms"], 3)}
            del o
        except RuntimeError as exc:  # backend not available for this shape / build
            res[name] = {"unavailable": str(exc).splitlines()[0][:160]}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
