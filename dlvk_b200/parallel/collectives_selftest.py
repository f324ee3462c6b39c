"""The NVLink backend's collectives (this framework's P2P kernels) against
NCCL's, one process per GPU:

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m dlvk_b200.parallel.collectives_selftest

Copies (broadcast, all-gather) must match exactly; sums (all-reduce,
reduce-scatter) to fp32 / bf16 rounding of a different summation order.
Prints one JSON line per rank."""
from __future__ import annotations

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def main() -> int:
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    from dlvk_b200 import _ext
    from dlvk_b200.parallel.comm import NcclBackend, NvlinkBackend

    nv, nc = NvlinkBackend(capacity_bytes=64 << 20), NcclBackend()
    assert nv.initialize()
    errs = {}
    for dt, tol in ((torch.float32, 1e-6), (torch.bfloat16, 1e-2)):
        for n in (1000, 4096 * world, (1 << 20) + 8 * world):
            g = torch.Generator(device="cuda").manual_seed(1000 * rank + n)
            x = torch.randn(n, device="cuda", generator=g).to(dt)
            a, b = x.clone(), x.clone()
            nv.broadcast(a, root=world - 1)
            nc.broadcast(b, root=world - 1)
            errs[f"broadcast_{dt}_{n}"] = float((a.float() - b.float()).abs().max())
            ga, gb = nv.all_gather(x), nc.all_gather(x)
            errs[f"all_gather_{dt}_{n}"] = max(float((p.float() - q.float()).abs().max()) for p, q in zip(ga, gb))
            a, b = x.clone(), x.clone()
            nv.all_reduce([a])
            nc.all_reduce([b])
            errs[f"all_reduce_{dt}_{n}"] = float((a.float() - b.float()).abs().max() / b.float().abs().max()) / tol
            if n % world == 0:
                ra, rb = nv.reduce_scatter(x), nc.reduce_scatter(x)
                errs[f"reduce_scatter_{dt}_{n}"] = float((ra.float() - rb.float()).abs().max() /
                                                         rb.float().abs().max()) / tol
    torch.cuda.synchronize()
    dev_err = int(_ext.C().read_device_error(True))
    copies_exact = all(v == 0.0 for k, v in errs.items() if k.startswith(("broadcast", "all_gather")))
    sums_close = all(v <= 1.0 for k, v in errs.items() if k.startswith(("all_reduce", "reduce_scatter")))
    ok = copies_exact and sums_close and dev_err == 0
    print(json.dumps({"rank": rank, "world": world, "ok": ok, "device_error": dev_err,
                      "worst": max(errs.items(), key=lambda kv: kv[1])}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
