"""Gradient all-reduce + Adam sweep (one process per GPU):

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m dlvk_b200.bench.allreduce [--dtype fp32|bf16]

For every bucket size (4 KB .. 1 GB of fp32 gradients) it times, on the
device (CUDA events around a CUDA graph of --iters steps, max over ranks):
  fused  this framework's one-kernel all-reduce + Adam (comm.cu), in the form
         the optimizer picks (LL one-shot for small buckets, pull two-shot,
         or push two-shot with --algo push); LL sizes also time the pull
         one-shot form, and --pull-ctas times two-shot at other grid sizes
  nccl   NCCL all-reduce followed by this framework's Adam kernel
and reports bus bandwidth (2 (N-1)/N * bytes / t, the all-reduce convention)
and the fused kernel's fraction of its roofline, max(bytes over NVLink per
direction / link bandwidth, local HBM bytes / measured HBM bandwidth).  The
link bandwidth is measured first: every rank copies 1 GiB from its
neighbour GPU at the same time (CUDA events, max over ranks), giving the
per-direction peer-copy rate under load; --nvlink-gbs overrides it.  With
NVLink multicast the two-shot sizes also time the NVLS form
(multimem.ld_reduce / multimem.st), whose link bytes are G/N in and V out
per rank for the reduce-scatter plus the multicast of V.  Byte counts:
  ll        NVLink 2 (N-1) * G;               HBM G + 2 (N-1) G + 24 n + V
  one-shot  NVLink (N-1) * G;                 HBM N*G + 24 n + V
  two-shot  NVLink (N-1)/N * (G + V);         HBM G + 24 n/N + V (pull),
                                              G (1 + 2 (N-1)/N) + 24 n/N + V (push)
for n elements, G = 4 n gradient bytes, V parameter bytes and 24 n/N the
fp32 master, m and v read and written by the shard owner.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dtype", default="bf16", choices=["fp32", "bf16"], help="parameter (compute) dtype")
    ap.add_argument("--min-kb", type=int, default=4)
    ap.add_argument("--max-mb", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--nvlink-gbs", type=float, default=0.0, help="0: measure the peer-copy rate")
    ap.add_argument("--pull-ctas", default="", help="comma list: also time the pull form at these grid sizes")
    ap.add_argument("--algo", default=None, choices=["auto", "pull", "push", "nvls"],
                    help="form (DLVK_AR_ALGO); auto: start-up calibration per size")
    ap.add_argument("--no-graph", dest="graph", action="store_false", help="time eager launches, not a CUDA graph")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    import dlvk_b200 as dl
    from dlvk_b200 import _ext
    from dlvk_b200.bench.common import measured_peaks
    from dlvk_b200.models.params import Parameter, ParamStore
    from dlvk_b200.parallel.comm import FusedAllReduceOptimizer

    C = _ext.C()
    hbm = measured_peaks()["hbm_gbs"] * 1e9
    link_gbs = args.nvlink_gbs
    if link_gbs <= 0:
        # every rank pulls 1 GiB from its neighbour at once (copy engines, NVLink)
        peer = (local + 1) % torch.cuda.device_count()
        src = torch.empty(1 << 28, dtype=torch.float32, device=f"cuda:{peer}")
        dst = torch.empty(1 << 28, dtype=torch.float32, device=f"cuda:{local}")
        for _ in range(3):
            dst.copy_(src)
        torch.cuda.synchronize(local)
        torch.cuda.synchronize(peer)
        dist.barrier()
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(5):
            dst.copy_(src)
        e0.record()
        torch.cuda.synchronize(local)
        t = torch.tensor([s0.elapsed_time(e0) / 5 / 1e3], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        link_gbs = (1 << 30) / float(t.item()) / 1e9
        del src, dst
        torch.cuda.empty_cache()
        if rank == 0:
            print(json.dumps({"peer_copy_gbs_per_direction": round(link_gbs, 1), "bytes": 1 << 30,
                              "method": "each rank copies 1 GiB from its neighbour GPU concurrently, "
                                        "CUDA events, max over ranks"}), flush=True)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    nmax = args.max_mb * (1 << 20) // 4
    g = torch.Generator().manual_seed(rank)
    p = Parameter("w", (nmax,), torch.randn(nmax, generator=g) * 0.02)
    store = ParamStore([p], f"cuda:{local}", dtype)
    opt = dl.Adam(1e-3)
    fused = FusedAllReduceOptimizer(store, opt, world, rank, algo=args.algo)
    store.grad.normal_(0, 1e-3)
    st = opt.state(store)
    sizes = []
    n = max(64, args.min_kb * 1024 // 4)
    while n <= nmax:
        sizes.append(n // 64 * 64)
        n *= 4

    def time_it(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        graph = None
        if args.graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(args.iters):
                    fn()
            graph.replay()  # untimed: the first replay uploads the graph
            torch.cuda.synchronize()
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(args.iters):
                fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del graph
        return float(t.item()) / 1e3

    for n in sizes:
        def fused_step(algo_override=None, ctas=None):
            fused.begin_step()
            opt.advance(store)
            fused.reduce_update(0, n, algo=algo_override, ctas=ctas)

        def nccl_step():
            gr = store.grad[:n]
            dist.all_reduce(gr)
            opt.advance(store)
            opt.update_range(store, 0, n, extra_scale=1.0 / world)

        algo = fused.algorithm(0, n)
        tf = time_it(fused_step)
        tpull = time_it(lambda: fused_step("pull")) if algo in ("push", "nvls") else None
        tnvls = None
        if fused.nvls and algo == "pull" and n * 4 > fused.one_shot_bytes:
            tnvls = time_it(lambda: fused_step("nvls"))
        toneshot = time_it(lambda: fused_step("one-shot")) if algo == "ll" else None
        tpull_ctas = {}
        if algo in ("push", "pull") and args.pull_ctas:
            for c in (int(v) for v in args.pull_ctas.split(",")):
                tpull_ctas[c] = time_it(lambda: fused_step("pull", c))
        tn = time_it(nccl_step)
        gbytes = n * 4
        vbytes = n * (2 if dtype == torch.bfloat16 else 4)
        state = 24 * n
        if algo == "ll":  # every rank stores 8 bytes per gradient to every peer
            link = (world - 1) * 2 * gbytes
            local_b = gbytes + (world - 1) * 2 * gbytes + state + vbytes
        elif algo == "one-shot":
            link = (world - 1) * gbytes
            local_b = world * gbytes + state + vbytes
        elif algo == "nvls":  # switch reduces; each rank sends G/N... in total G out, V/N x N copies in
            link = max(gbytes, (world - 1) / world * vbytes + gbytes / world)
            local_b = gbytes + state / world + vbytes
        else:
            link = (world - 1) / world * (gbytes + vbytes)
            local_b = gbytes * (1 + (2 * (world - 1) / world if algo == "push" else 0)) + state / world + vbytes
        roof = max(link / (link_gbs * 1e9), local_b / hbm)
        bus = 2 * (world - 1) / world * gbytes
        if rank == 0:
            row = {"world": world, "bucket_bytes": gbytes, "param_dtype": args.dtype, "algo": algo,
                   "timing": "cuda-graph" if args.graph else "eager",
                   "fused_us": round(tf * 1e6, 1), "nccl_plus_adam_us": round(tn * 1e6, 1),
                   "fused_bus_gbs": round(bus / tf / 1e9, 1), "nccl_bus_gbs": round(bus / tn / 1e9, 1),
                   "fused_roofline_us": round(roof * 1e6, 1),
                   "fused_frac_of_roofline": round(roof / tf, 3),
                   "speedup_vs_nccl_plus_adam": round(tn / tf, 3)}
            row["link_gbs_per_direction"] = round(link_gbs, 1)
            if tpull is not None:
                row["pull_us"] = round(tpull * 1e6, 1)
            if tnvls is not None:
                row["nvls_us"] = round(tnvls * 1e6, 1)
                row["nvls_bus_gbs"] = round(bus / tnvls / 1e9, 1)
            if toneshot is not None:
                row["pull_one_shot_us"] = round(toneshot * 1e6, 1)
            for c, t in tpull_ctas.items():
                row[f"pull_{c}ctas_us"] = round(t * 1e6, 1)
            print(json.dumps(row), flush=True)
    err = C.read_device_error(True)
    if rank == 0:
        print(json.dumps({"device_error": int(err), "nvls": fused.nvls if fused.nvls else fused.nvls_reason,
                          "calibration_us": (fused.calibration or {}).get("us")}))
    fused.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
