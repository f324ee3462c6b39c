"""GEMM micro-benchmark: the tcgen05 kernel against cuBLAS (torch.matmul) on
the shapes of the transformer and wide-MLP training steps.

    python -m dlvk_b200.bench.gemm [--shapes M,N,K ...] [--iters 20]
"""
from __future__ import annotations

import argparse
import json

import torch

from dlvk_b200 import _ext
from dlvk_b200.bench.common import measured_peaks, time_fn

DEFAULT = [
    # (M, N, K, a_major, b_major): 'k' = K-major, 'mn' = M/N-major
    (8192, 3072, 1024, "k", "mn"),   # QKV projection  X @ W
    (8192, 4096, 1024, "k", "mn"),   # FFN up
    (8192, 1024, 4096, "k", "mn"),   # FFN down
    (8192, 1024, 4096, "k", "k"),    # dX = dY @ W^T
    (1024, 4096, 8192, "mn", "mn"),  # dW = X^T @ dY
    (8192, 32000, 1024, "k", "mn"),  # vocab projection
    (1024, 4096, 4096, "k", "mn"),   # wide MLP layer
    (8192, 8192, 8192, "k", "mn"),
]


def make(M, N, K, am, bm):
    a = torch.randn(M, K, device="cuda").bfloat16() if am == "k" else torch.randn(K, M, device="cuda").bfloat16().t()
    b = torch.randn(K, N, device="cuda").bfloat16() if bm == "mn" else torch.randn(N, K, device="cuda").bfloat16().t()
    return a, b


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-flush", action="store_true",
                    help="back-to-back launches with L2 warm (as inside a training step), not L2 flushed before each")
    ap.add_argument("--shapes", nargs="*", default=None)
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--bias", action="store_true", help="fp32 bias in the epilogue")
    ap.add_argument("--relu", action="store_true", help="ReLU in the epilogue")
    ap.add_argument("--residual", action="store_true", help="residual add in the epilogue")
    ap.add_argument("--mask", action="store_true", help="ReLU-mask input in the epilogue")
    ap.add_argument("--out-f32", action="store_true",
                    help="fp32 output, as for weight gradients (cuBLAS still writes bf16)")
    ap.add_argument("--beta", type=float, default=0.0, help="accumulate: C = A B + beta C")
    ap.add_argument("--wide", type=int, default=1,
                    help="256 x 512 pair tile: 0 never, 1 when the tiling model picks it, 2 whenever it applies")
    ap.add_argument("--compare-single", action="store_true",
                    help="also time the single-CTA kernel (CTA-pair variant switched off)")
    ap.add_argument("--tilings", default="",
                    help="semicolon list of bn,splits,pair to time besides the model's choice, e.g. '256,2,1;128,2,0'")
    ap.add_argument("--fp32", action="store_true",
                    help="fp32 operands: ours 3xTF32 and 1xTF32 against cuBLAS TF32 and cuBLAS fp32")
    args = ap.parse_args()
    if args.fp32:
        return fp32_main(args)
    C = _ext.C()
    C.gemm_set_wide(args.wide)
    shapes = DEFAULT
    if args.shapes:
        shapes = []
        for s in args.shapes:
            p = s.split(",")
            shapes.append((int(p[0]), int(p[1]), int(p[2]), p[3] if len(p) > 3 else "k", p[4] if len(p) > 4 else "mn"))
    peak = measured_peaks()["bf16_tflops"]
    for (M, N, K, am, bm) in shapes:
        a, b = make(M, N, K, am, bm)
        out = torch.zeros(M, N, device="cuda", dtype=torch.float32 if args.out_f32 else torch.bfloat16)
        out_cb = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * M * N * K
        kw = {}
        if args.bias:
            kw["bias"] = torch.randn(N, device="cuda")
        if args.relu:
            kw["act"] = 1
        if args.residual:
            kw["residual"] = torch.randn(M, N, device="cuda").bfloat16()
        if args.mask:
            kw["relu_mask"] = torch.randn(M, N, device="cuda").bfloat16()
        if args.beta:
            kw["beta"] = args.beta
        t_ours = time_fn(lambda: C.gemm(a, b, out=out, force_path=1, **kw), iters=args.iters, flush=not args.no_flush)
        rec = {"M": M, "N": N, "K": K, "a": am, "b": bm, "epilogue": sorted(kw), "out": str(out.dtype)[6:],
               "plan": list(C.gemm_plan(a, b, args.out_f32)),
               "ours_ms": round(t_ours, 4),
               "ours_tflops": round(flops / t_ours / 1e9, 1), "ours_frac_of_measured": round(flops / t_ours / 1e9 / peak, 3)}
        for tl in [t for t in args.tilings.split(";") if t]:
            bn, sp, pr = (int(v) for v in tl.split(","))
            C.gemm_set_tiling(bn, sp, pr)
            try:
                tt = time_fn(lambda: C.gemm(a, b, out=out, force_path=1, **kw), iters=args.iters, flush=not args.no_flush)
                ref = a.float() @ b.float()
                C.gemm(a, b, out=out, force_path=1, **kw)
                ok = float((out.float() - ref).abs().max() / ref.abs().max()) < 2e-2
            finally:
                C.gemm_set_tiling(0, 0, -1)
            rec[f"tiling_{bn}_{sp}_{pr}_ms"] = round(tt, 4) if ok else "wrong"
        if args.compare_single:
            C.gemm_set_pair(False)
            try:
                t_1 = time_fn(lambda: C.gemm(a, b, out=out, force_path=1, **kw), iters=args.iters, flush=not args.no_flush)
            finally:
                C.gemm_set_pair(True)
            rec.update({"single_cta_ms": round(t_1, 4), "single_cta_tflops": round(flops / t_1 / 1e9, 1)})
        if not args.no_cublas:
            t_cb = time_fn(lambda: torch.matmul(a, b, out=out_cb), iters=args.iters, flush=not args.no_flush)
            rec.update({"cublas_ms": round(t_cb, 4), "cublas_tflops": round(flops / t_cb / 1e9, 1),
                        "speedup_vs_cublas": round(t_cb / t_ours, 3)})
        if args.check:
            ref = a.float() @ b.float()
            C.gemm(a, b, out=out, force_path=1)
            rec["max_rel_err"] = float((out.float() - ref).abs().max() / ref.abs().max())
        print(json.dumps(rec), flush=True)


def fp32_main(args):
    """fp32 GEMMs: the tcgen05 kind::tf32 path (three passes with the 3xTF32
    split, and one pass) against cuBLAS with TF32 allowed and with full fp32;
    error against an fp64 product of the same operands."""
    C = _ext.C()
    shapes = [(8192, 4096, 4096, "k", "mn"), (4096, 4096, 4096, "k", "mn"), (1024, 4096, 8192, "mn", "mn")]
    if args.shapes:
        shapes = [tuple(int(v) if i < 3 else v for i, v in enumerate(s.split(","))) for s in args.shapes]
    peak = measured_peaks()["bf16_tflops"]
    old_mode = C.fp32_gemm_mode()
    for (M, N, K, am, bm) in shapes:
        a = torch.randn(M, K, device="cuda") if am == "k" else torch.randn(K, M, device="cuda").t()
        b = torch.randn(K, N, device="cuda") if bm == "mn" else torch.randn(N, K, device="cuda").t()
        out = torch.empty(M, N, device="cuda")
        flops = 2.0 * M * N * K
        ref = a.double() @ b.double()
        rec = {"M": M, "N": N, "K": K, "a": am, "b": bm}
        for name, mode in (("ours_3xtf32", 3), ("ours_tf32", 1)):
            C.set_fp32_gemm_mode(mode)
            t = time_fn(lambda: C.gemm(a, b, out=out, force_path=1), iters=args.iters, flush=not args.no_flush)
            rec[name + "_ms"] = round(t, 4)
            rec[name + "_tflops"] = round(flops / t / 1e9, 1)
            rec[name + "_rel_err"] = float((out.double() - ref).norm() / ref.norm())
        C.set_fp32_gemm_mode(old_mode)
        for name, tf in (("cublas_tf32", True), ("cublas_fp32", False)):
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = tf
            try:
                t = time_fn(lambda: torch.matmul(a, b, out=out), iters=args.iters, flush=not args.no_flush)
                rec[name + "_ms"] = round(t, 4)
                rec[name + "_tflops"] = round(flops / t / 1e9, 1)
                rec[name + "_rel_err"] = float((out.double() - ref).norm() / ref.norm())
            finally:
                torch.backends.cuda.matmul.allow_tf32 = prev
        rec["ours_3xtf32_vs_cublas_fp32"] = round(rec["cublas_fp32_ms"] / rec["ours_3xtf32_ms"], 3)
        rec["ours_tf32_vs_cublas_tf32"] = round(rec["cublas_tf32_ms"] / rec["ours_tf32_ms"], 3)
        rec["bf16_peak_tflops_measured"] = peak
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
