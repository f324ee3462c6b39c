"""Data-parallel self-test: N ranks train a model on disjoint shards of one
batch; the result must equal single-process training on the whole batch.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m dlvk_b200.parallel.selftest --mode fused --model mlp

Each rank checks its parameters against a reference it computes itself on
the full batch (same seed, same initial weights), prints one JSON line and
exits non-zero on mismatch.  Works on CPU with gloo (mode nccl) as well.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--model", default="mlp", choices=["mlp", "transformer"])
    ap.add_argument("--dtype", default="fp32")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--bucket-mb", type=float, default=0.05)
    ap.add_argument("--one-shot-bytes", type=int, default=None)
    ap.add_argument("--ll", type=int, default=1, help="0: small buckets use the pull one-shot form, not LL")
    ap.add_argument("--algo", default=None, choices=["auto", "push", "pull", "nvls"],
                    help="form of the fused path (auto: calibrated per bucket size)")
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--fail-rank", type=int, default=-1,
                    help="fault injection on the host: this rank exits between steps")
    ap.add_argument("--fail-step", type=int, default=1)
    ap.add_argument("--pg-timeout", type=float, default=60.0)
    ap.add_argument("--tol", type=float, default=None)
    ap.add_argument("--opt", default="adam", choices=["adam", "sgd"],
                    help="sgd keeps bf16 rounding differences linear; Adam maps near-zero "
                         "gradients of either sign to +-lr on its first step")
    args = ap.parse_args()

    import dlvk_b200 as dl
    from dlvk_b200.models import zoo
    from dlvk_b200.parallel.data_parallel import DataParallel
    from dlvk_b200.training.step import TrainStep

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.cpu:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=args.pg_timeout))
        device = "cpu"
    else:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=args.pg_timeout),
                                device_id=torch.device("cuda", local))
        device = f"cuda:{local}"
    if args.one_shot_bytes is not None:
        os.environ["DLVK_ONE_SHOT_BYTES"] = str(args.one_shot_bytes)
    if args.algo is not None:
        os.environ["DLVK_AR_ALGO"] = args.algo
    os.environ["DLVK_AR_LL"] = str(args.ll)

    def build(dev):
        if args.model == "mlp":
            return zoo.mlp(device=dev, dtype=args.dtype, seed=0)
        return zoo.transformer(device=dev, dtype=args.dtype, seed=0, vocab=256, d_model=128, layers=2, heads=2,
                               d_ff=256)

    per = 8
    g = torch.Generator().manual_seed(123)
    if args.model == "mlp":
        X = torch.rand(per * world, 784, generator=g)
        Y = torch.randint(0, 10, (per * world,), generator=g, dtype=torch.int32)
    else:
        toks = torch.randint(0, 256, (per * world, 33), generator=g, dtype=torch.int32)
        X, Y = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()

    # reference: one process, full batch (mean over all rows == DP mean of shard means)
    ref = build(device)
    make_opt = (lambda: dl.Adam(1e-2)) if args.opt == "adam" else (lambda: dl.SGD(0.05, momentum=0.9))
    ref_opt = make_opt()
    ref_step = TrainStep(ref, dl.CrossEntropyLoss(), ref_opt, graph=False)
    for _ in range(args.steps):
        ref_step(X, Y)

    model = build(device)
    opt = make_opt()
    dp = DataParallel(model, opt, mode=args.mode, bucket_mb=args.bucket_mb)
    step = TrainStep(model, dl.CrossEntropyLoss(), opt, dp=dp, graph=False)
    xs, ys = X[rank * per:(rank + 1) * per].contiguous(), Y[rank * per:(rank + 1) * per].contiguous()
    for it in range(args.steps):
        if rank == args.fail_rank and it == args.fail_step:
            # leaves between steps: nothing of this rank is in flight
            print(json.dumps({"rank": rank, "injected_exit": it}), flush=True)
            os._exit(3)
        try:
            loss = step(xs, ys)
        except Exception as e:  # a peer left: the collective fails instead of hanging
            print(json.dumps({"rank": rank, "peer_failure_detected": True, "step": it,
                              "error": type(e).__name__}), flush=True)
            os._exit(4)
    dp.consolidate()
    if not args.cpu:
        torch.cuda.synchronize()
    err_word = 0
    if not args.cpu:
        from dlvk_b200 import _ext

        err_word = int(_ext.C().read_device_error(True))
    a = model.store.value.float()
    b = ref.store.value.float()
    diff = float((a - b).abs().max())
    scale = float(b.abs().max())
    tol = args.tol if args.tol is not None else (2e-4 if args.dtype == "fp32" else 2e-2)
    ok = diff <= tol * scale and err_word == 0
    mdiff = float((model.store.master - ref.store.master).abs().max())
    res = {"rank": rank, "world": world, "mode": args.mode, "model": args.model, "dtype": args.dtype,
           "max_param_diff": diff, "param_scale": scale, "master_diff": mdiff, "device_error": err_word,
           "buckets": dp.describe()["buckets"], "forms": dp.describe().get("forms"), "ok": ok,
           "loss": float(loss)}
    print(json.dumps(res), flush=True)
    dp.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
