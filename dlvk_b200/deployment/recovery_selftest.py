"""Restart-from-checkpoint check for data-parallel training (the reference's
MultiGPUTrainer::save_checkpoint / load_checkpoint,
src/deployment/multi_gpu_trainer.cpp:144-156, which were stubs).

One phase per launch, every rank of a torchrun job:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m dlvk_b200.deployment.recovery_selftest --phase first --dir D [--cpu]

  full    train steps 0 .. total-1 without interruption, save D/full.dlvk
  first   train steps 0 .. split-1, save the checkpoint D/ckpt.dlvk, exit
  resume  new processes: build a freshly initialised model, load
          D/ckpt.dlvk (weights, optimizer state, step counters) on every
          rank, train steps split .. total-1, save D/resumed.dlvk

The batch of step i on rank r depends only on (i, r), so a resumed run sees
the same data as the uninterrupted one; D/resumed.dlvk must equal
D/full.dlvk byte for byte.  With --cpu the ranks run on gloo.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def _batch(step: int, rank: int, per: int = 8):
    g = torch.Generator().manual_seed(1000 * step + rank)
    return torch.rand(per, 784, generator=g), torch.randint(0, 10, (per,), generator=g, dtype=torch.int32)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--phase", required=True, choices=["full", "first", "resume"])
    ap.add_argument("--dir", required=True)
    ap.add_argument("--total", type=int, default=5)
    ap.add_argument("--split", type=int, default=3)
    ap.add_argument("--cpu", action="store_true")
    args = ap.parse_args()

    import dlvk_b200 as dl
    from dlvk_b200.deployment.multi_gpu import MultiGPUConfig, MultiGPUTrainer
    from dlvk_b200.models import zoo

    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.cpu:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
        device = "cpu"
    else:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", local))
        device = f"cuda:{local}"
    rank = dist.get_rank()

    cfg = MultiGPUConfig()
    cfg.use_nccl = args.cpu  # the fused peer-memory path needs GPUs
    trainer = MultiGPUTrainer(cfg)
    # a different initial seed for the resumed job: its weights must come
    # from the checkpoint, not from initialisation
    model = zoo.mlp(device=device, dtype="fp32", seed=0 if args.phase != "resume" else 99)
    trainer.initialize(model, dl.Adam(1e-3), dl.CrossEntropyLoss())

    if args.phase == "resume":
        trainer.load_checkpoint(os.path.join(args.dir, "ckpt.dlvk"))
        steps = range(args.split, args.total)
    elif args.phase == "first":
        steps = range(0, args.split)
    else:
        steps = range(0, args.total)
    trainer.train([_batch(i, rank) for i in steps], epochs=1)
    name = {"full": "full.dlvk", "first": "ckpt.dlvk", "resume": "resumed.dlvk"}[args.phase]
    trainer.save_checkpoint(os.path.join(args.dir, name))
    print(json.dumps({"rank": rank, "phase": args.phase, "steps": list(steps), "ok": True}), flush=True)
    trainer.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
