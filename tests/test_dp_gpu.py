"""Fused NVLink all-reduce + optimizer on 2+ GPUs against single-process
full-batch training (and the NCCL path)."""
import pytest
import torch

from test_dp_cpu import run_selftest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("model,dtype,oneshot,opt,algo", [("mlp", "fp32", 1 << 30, "adam", "auto"),
                                                          ("mlp", "fp32", 1 << 30, "adam", "noll"),
                                                          ("transformer", "bf16", 1 << 30, "sgd", "noll"),
                                                          ("mlp", "fp32", 0, "adam", "push"),
                                                          ("mlp", "fp32", 0, "adam", "pull"),
                                                          ("transformer", "bf16", 1 << 30, "sgd", "auto"),
                                                          ("transformer", "bf16", 0, "sgd", "push"),
                                                          ("transformer", "bf16", 0, "sgd", "pull"),
                                                          ("transformer", "fp32", 0, "adam", "push")])
def test_fused_dp_matches_full_batch(model, dtype, oneshot, opt, algo):
    _need(2)
    extra = ["--ll", "0"] if algo == "noll" else ["--algo", algo]
    rc, lines, log = run_selftest(2, ["--mode", "fused", "--model", model, "--dtype", dtype,
                                      "--one-shot-bytes", str(oneshot), "--opt", opt] + extra)
    assert rc == 0, log[-4000:]
    assert len(lines) == 2 and all(l["ok"] for l in lines), lines


# Every fused form at 2, 4 and 8 ranks (the kernels are instantiated per
# world size) against single-process full-batch training.  "nvls" needs
# NVLink multicast; "auto" runs the start-up calibration and its choices.
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("model,dtype,oneshot,opt,algo", [("mlp", "fp32", 1 << 30, "adam", "auto"),
                                                          ("mlp", "fp32", 1 << 30, "adam", "noll"),
                                                          ("mlp", "fp32", 0, "adam", "pull"),
                                                          ("mlp", "fp32", 0, "adam", "push"),
                                                          ("mlp", "fp32", 0, "adam", "nvls"),
                                                          ("transformer", "bf16", 0, "sgd", "nvls"),
                                                          ("transformer", "bf16", 0, "sgd", "auto")])
def test_fused_dp_forms_at_world(world, model, dtype, oneshot, opt, algo):
    _need(world)
    extra = ["--ll", "0"] if algo == "noll" else ["--algo", algo]
    rc, lines, log = run_selftest(world, ["--mode", "fused", "--model", model, "--dtype", dtype,
                                          "--one-shot-bytes", str(oneshot), "--opt", opt] + extra)
    if algo == "nvls" and "NVLS all-reduce requested but unavailable" in log:
        pytest.skip("no NVLink multicast on this node")
    assert rc == 0, log[-4000:]
    assert len(lines) == world and all(l["ok"] for l in lines), lines
    if algo == "nvls":
        assert all("nvls" in (l.get("forms") or []) for l in lines), lines


def test_nccl_dp_matches_full_batch():
    _need(2)
    rc, lines, log = run_selftest(2, ["--mode", "nccl", "--model", "transformer", "--dtype", "bf16", "--opt", "sgd"])
    assert rc == 0, log[-4000:]
    assert all(l["ok"] for l in lines), lines


@pytest.mark.parametrize("extra", [[], ["--nccl"]])
def test_multi_gpu_trainer_api(extra):
    """MultiGPUTrainer + RingAllReduce (P2P kernel) on 2 GPUs."""
    import os
    import subprocess
    import sys

    from test_dp_cpu import ROOT, _port, parse_objects

    _need(2)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", f"--master-port={_port()}", "-m", "dlvk_b200.deployment.selftest"] + extra
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    res = parse_objects(r.stdout)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert len(res) == 2 and all(o["ok"] for o in res), res


def test_nvlink_backend_collectives_match_nccl():
    """broadcast / all_gather / reduce_scatter / all_reduce on this
    framework's P2P kernels against NCCL, 2 ranks."""
    import os
    import subprocess
    import sys

    from test_dp_cpu import ROOT, _port, parse_objects

    _need(2)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", f"--master-port={_port()}", "-m", "dlvk_b200.parallel.collectives_selftest"]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    res = parse_objects(r.stdout)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert len(res) == 2 and all(o["ok"] for o in res), res
