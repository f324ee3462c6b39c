"""Memory-bound kernel micro-benchmark at the transformer config's shapes
(8192 rows = batch 16 x seq 512, d_model 1024, vocab 32000, bf16): LayerNorm
forward and backward (with the residual gradient), fused softmax +
cross-entropy, bias-gradient column sums and the Adam update, plus the
wide-MLP config's BatchNorm1D (+ ReLU + dropout 0.1) forward and backward on
[1024, 4096]; each as achieved GB/s of its algorithmic bytes and the fraction
of the measured HBM copy bandwidth.  CUDA-event timed, L2 flushed between
launches.

    python -m dlvk_b200.bench.kernels [--rows 8192 --d 1024 --vocab 32000] [--only bn]
"""
from __future__ import annotations

import argparse
import json

import torch

from dlvk_b200.bench.common import measured_peaks, time_fn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--d", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--params", type=int, default=185_000_000)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default=None, choices=["bn", "ce", "ln"],
                    help="bn: only the BatchNorm rows; ce: only softmax + cross-entropy; ln: only LayerNorm")
    a = ap.parse_args()
    import dlvk_b200 as dl
    from dlvk_b200.models.params import Parameter, ParamStore
    from dlvk_b200.ops import core as K
    from dlvk_b200.ops import nn as NN

    hbm = measured_peaks()["hbm_gbs"] * 1e9
    R, D, V = a.rows, a.d, a.vocab
    x = torch.randn(R, D, device="cuda").bfloat16()
    dy = torch.randn(R, D, device="cuda").bfloat16()
    dres = torch.randn(R, D, device="cuda").bfloat16()
    gamma = torch.ones(D, device="cuda")
    beta = torch.zeros(D, device="cuda")
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    rows = []

    def report(name, t_ms, nbytes):
        t = t_ms * 1e-3
        rows.append({"kernel": name, "us": round(t * 1e6, 2), "gbs": round(nbytes / t / 1e9, 1),
                     "frac_of_measured_hbm": round(nbytes / t / hbm, 3)})

    def want(g):
        return a.only is None or a.only == g

    if want("bn"):
        bx = torch.randn(1024, 4096, device="cuda").bfloat16()
        bg = torch.randn(1024, 4096, device="cuda").bfloat16()
        bgam, bbet = torch.rand(4096, device="cuda") + 0.5, torch.randn(4096, device="cuda") * 0.1
        rmean, rvar = torch.zeros(4096, device="cuda"), torch.ones(4096, device="cuda")
        dgb, dbb = torch.zeros(4096, device="cuda"), torch.zeros(4096, device="cuda")
        _, bm, bs = NN.batchnorm_fwd(bx, bgam, bbet, rmean, rvar, 0.1, 1e-5, True, True, 0.1, 3, 7, 5)
        n = bx.numel()
        report("batchnorm1d_fwd+relu+dropout [1024,4096]",
               time_fn(lambda: NN.batchnorm_fwd(bx, bgam, bbet, rmean, rvar, 0.1, 1e-5, True, True, 0.1, 3, 7, 5),
                       a.iters), 2 * n * 2)  # read x, write y (the second read of x hits L2)
        report("batchnorm1d_bwd+relu+dropout [1024,4096]",
               time_fn(lambda: NN.batchnorm_bwd(bx, bg, bm, bs, bgam, bbet, dgb, dbb, False, True, 0.1, 3, 7, 5),
                       a.iters), 3 * n * 2)  # read x and dy, write dx
    if a.only == "bn":
        for r in rows:
            print(json.dumps(r), flush=True)
        return
    if a.only == "ce":
        logits = torch.randn(R, V, device="cuda").bfloat16()
        tgt = torch.randint(0, V, (R,), device="cuda", dtype=torch.int32)
        report("softmax_ce(+grad in place)", time_fn(lambda: K.softmax_ce(logits, tgt, 1.0 / R, True, True), a.iters),
               2 * R * V * 2)
        for r in rows:
            print(json.dumps(r), flush=True)
        return
    # Same-size anchors on the same box: a plain device copy of x (read 16 MB,
    # write 16 MB) and PyTorch's own LayerNorm forward / backward.
    yc = torch.empty_like(x)
    report("[anchor] copy x -> y (torch)", time_fn(lambda: yc.copy_(x), a.iters), 2 * R * D * 2)
    xt = x.detach().clone().requires_grad_(True)
    gt = gamma.detach().bfloat16().requires_grad_(True)  # torch wants the input's dtype
    bt = beta.detach().bfloat16().requires_grad_(True)
    report("[anchor] layernorm_fwd (torch)",
           time_fn(lambda: torch.nn.functional.layer_norm(x, (D,), gt.detach(), bt.detach(), 1e-5), a.iters),
           2 * R * D * 2 + R * 8)
    yt = torch.nn.functional.layer_norm(xt, (D,), gt, bt, 1e-5)
    report("[anchor] layernorm_bwd (torch)",
           time_fn(lambda: torch.autograd.grad(yt, (xt, gt, bt), dy, retain_graph=True), a.iters),
           3 * R * D * 2 + R * 8)
    y, mean, rstd = NN.layernorm_fwd(x, gamma, beta, 1e-5)
    report("layernorm_fwd", time_fn(lambda: NN.layernorm_fwd(x, gamma, beta, 1e-5), a.iters), 2 * R * D * 2 + R * 8)
    report("layernorm_bwd+dres", time_fn(lambda: NN.layernorm_bwd(x, gamma, mean, rstd, dy, dg, db, False, dres),
                                          a.iters), 4 * R * D * 2 + R * 8)
    report("layernorm_bwd", time_fn(lambda: NN.layernorm_bwd(x, gamma, mean, rstd, dy, dg, db, False), a.iters),
           3 * R * D * 2 + R * 8)
    if a.only == "ln":
        for r in rows:
            print(json.dumps(r), flush=True)
        return
    logits = torch.randn(R, V, device="cuda").bfloat16()
    tgt = torch.randint(0, V, (R,), device="cuda", dtype=torch.int32)
    report("softmax_ce(+grad in place)", time_fn(lambda: K.softmax_ce(logits, tgt, 1.0 / R, True, True), a.iters),
           2 * R * V * 2)
    g4 = torch.randn(R, 4 * D, device="cuda").bfloat16()
    report("colsum [8192,4096]", time_fn(lambda: K.colsum(g4, 1.0), a.iters), R * 4 * D * 2)
    p = Parameter("w", (a.params,), torch.zeros(a.params))
    store = ParamStore([p], "cuda:0", torch.bfloat16)
    store.grad.normal_()
    opt = dl.Adam(1e-3)
    opt.state(store)
    opt.advance(store)
    report("adam_update", time_fn(lambda: opt.update_range(store, 0, a.params), a.iters),
           a.params * (4 + 8 + 8 + 8 + 2))
    for r in rows:
        print(json.dumps(r), flush=True)
    from dlvk_b200 import _ext

    print(json.dumps({"device_error": int(_ext.C().read_device_error(True))}))


if __name__ == "__main__":
    main()
