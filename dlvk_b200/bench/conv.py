"""Convolution micro-benchmark, bf16: the implicit-GEMM tcgen05 kernels
(conv_tc.cu, layout copies and weight packing included) against this
framework's direct kernels and PyTorch's cuDNN convolution, forward, dgrad and
wgrad, CUDA-event timed with L2 flushed between launches.

    python -m dlvk_b200.bench.conv [--iters 20] [--shapes N,C,H,W,OC,k,s,p ...]
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

from dlvk_b200.bench.common import measured_peaks, time_fn

DEFAULT = ["32,64,56,56,64,3,1,1", "32,128,28,28,128,3,1,1", "32,256,14,14,256,3,1,1", "64,64,56,56,256,1,1,0",
           "256,8,14,14,16,3,1,1"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--shapes", nargs="*", default=DEFAULT)
    ap.add_argument("--no-direct", action="store_true", help="skip the direct kernels (slow on wide layers)")
    a = ap.parse_args()
    from dlvk_b200 import _ext

    C = _ext.C()
    peak = measured_peaks()["bf16_tflops"] * 1e12
    old = C.conv_tc_get_mode()
    for spec in a.shapes:
        N, Cin, H, W, Cout, k, s, p = (int(v) for v in spec.split(","))
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        x = torch.randn(N, Cin, H, W, device="cuda").bfloat16()
        w = (torch.randn(Cout, Cin, k, k, device="cuda") * 0.05).bfloat16()
        b = torch.randn(Cout, device="cuda")
        gy = torch.randn(N, Cout, Ho, Wo, device="cuda").bfloat16()
        dw = torch.zeros(Cout, Cin, k, k, device="cuda")
        flops = 2.0 * N * Ho * Wo * Cout * Cin * k * k
        row = {"shape": spec, "gflop_per_pass": round(flops / 1e9, 3),
               "tc_path": Cin % 8 == 0 and Cout % 8 == 0 and Cin >= 16 and Cout >= 16}
        modes = [("tc", 1)] + ([] if a.no_direct else [("direct", 2)])
        for name, mode in modes:
            C.conv_tc_set_mode(mode)
            for part, fn in (("fwd", lambda: C.conv2d_fwd(x, w, b, s, p, False)),
                             ("dgrad", lambda: C.conv2d_dgrad(gy, w, [N, Cin, H, W], s, p, None)),
                             ("wgrad", lambda: C.conv2d_wgrad(x, gy, dw, None, s, p, False))):
                try:
                    t = time_fn(fn, a.iters) * 1e-3  # seconds
                except RuntimeError as e:  # a direct kernel's size limit
                    row[f"{name}_{part}_us"] = f"unsupported: {str(e).splitlines()[0][:80]}"
                    continue
                row[f"{name}_{part}_us"] = round(t * 1e6, 1)
                row[f"{name}_{part}_tflops"] = round(flops / t / 1e12, 1)
                row[f"{name}_{part}_frac_of_measured_peak"] = round(flops / t / peak, 3)
        C.conv_tc_set_mode(old)
        wf = w.float().bfloat16()
        tf = time_fn(lambda: F.conv2d(x, wf, b.bfloat16(), stride=s, padding=p), a.iters)
        td = time_fn(lambda: torch.nn.grad.conv2d_input([N, Cin, H, W], wf, gy, stride=s, padding=p), a.iters)
        tw = time_fn(lambda: torch.nn.grad.conv2d_weight(x, [Cout, Cin, k, k], gy, stride=s, padding=p), a.iters)
        row["cudnn_fwd_us"] = round(tf * 1e3, 1)
        row["cudnn_dgrad_us"] = round(td * 1e3, 1)
        row["cudnn_wgrad_us"] = round(tw * 1e3, 1)
        print(json.dumps(row), flush=True)
    print(json.dumps({"device_error": int(C.read_device_error(True))}))


if __name__ == "__main__":
    main()
