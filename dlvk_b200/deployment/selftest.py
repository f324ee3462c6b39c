"""Multi-process check of MultiGPUTrainer / RingAllReduce:

    torchrun --nproc-per-node 2 -m dlvk_b200.deployment.selftest [--cpu]

Every rank trains on its shard of one synthetic classification set; the
ranks' weights must stay identical, the loss must fall, and the ring
all-reduce must return the element-wise sum.  Prints one JSON line per rank."""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cpu", action="store_true")
    ap.add_argument("--nccl", action="store_true", help="NCCL all-reduce + optimizer instead of the fused kernel")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    from datetime import timedelta

    if a.cpu:
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        dev = "cpu"
    else:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
        dev = f"cuda:{torch.cuda.current_device()}"
    from .. import losses as Lo
    from .. import optim as O
    from ..data import DataLoader, TensorDataset
    from ..models.sequential import Sequential
    from .multi_gpu import MultiGPUConfig, MultiGPUTrainer, RingAllReduce

    g = torch.Generator().manual_seed(0)
    C = torch.randn(10, 32, generator=g) * 3
    y = torch.randint(0, 10, (2048,), generator=g)
    x = C[y] + torch.randn(2048, 32, generator=g)
    ds = TensorDataset(x, y.to(torch.int32), 10)
    dl = DataLoader(ds, dev if not a.cpu else None, batch_size=128, one_hot=False, rank=rank, world_size=world)
    m = Sequential(dev, "fp32", seed=rank)  # different init per rank: the trainer must broadcast rank 0's
    m.add_dense(32, 64).add_relu().add_dense(64, 10).add_softmax()
    m.build()
    tr = MultiGPUTrainer(MultiGPUConfig(use_nccl=a.nccl or a.cpu))
    tr.initialize(m, O.SGD(0.05, momentum=0.9), Lo.CrossEntropyLoss())
    first = tr.evaluate(dl).loss
    met = tr.train(dl, epochs=3)
    w = tr.get_consolidated_model().store.master.clone()
    ws = [torch.empty_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    same = all(torch.equal(ws[0], v) for v in ws)
    ring = RingAllReduce(use_p2p=not a.cpu)
    t = torch.full((1000,), float(rank + 1), device=dev)
    ring.perform_all_reduce([t])
    ring_ok = bool(torch.all(t == world * (world + 1) / 2))
    st = tr.get_stats()
    res = {"rank": rank, "ok": bool(same and met.loss < first and ring_ok), "same_weights": same,
           "loss0": first, "loss": met.loss, "acc": met.accuracy, "ring_ok": ring_ok,
           "batches": st.total_batches, "ring_gbps": ring.get_stats().bandwidth_gbps}
    print(json.dumps(res), flush=True)
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
