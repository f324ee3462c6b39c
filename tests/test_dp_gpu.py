"""Fused NVLink all-reduce + optimizer on 2+ GPUs against single-process
full-batch training (and the NCCL path)."""
import pytest
import torch

from test_dp_cpu import run_selftest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("model,dtype,oneshot", [("mlp", "fp32", 1 << 30), ("mlp", "fp32", 0),
                                                 ("transformer", "bf16", 1 << 30), ("transformer", "bf16", 0),
                                                 ("transformer", "fp32", 0)])
def test_fused_dp_matches_full_batch(model, dtype, oneshot):
    _need(2)
    rc, lines, log = run_selftest(2, ["--mode", "fused", "--model", model, "--dtype", dtype,
                                      "--one-shot-bytes", str(oneshot)])
    assert rc == 0, log[-4000:]
    assert len(lines) == 2 and all(l["ok"] for l in lines), lines


def test_nccl_dp_matches_full_batch():
    _need(2)
    rc, lines, log = run_selftest(2, ["--mode", "nccl", "--model", "transformer", "--dtype", "bf16"])
    assert rc == 0, log[-4000:]
    assert all(l["ok"] for l in lines), lines
