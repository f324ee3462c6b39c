"""Failure detection without a GPU fault: host-side fault injection on gloo
ranks, checkpoint-write failures, the device error word, and (on a GPU) the
bounded peer wait of the all-reduce kernels running out on a flag that
nothing sets."""
import os
import subprocess
import sys
import time

import pytest
import torch

sys.path.insert(0, os.path.dirname(__file__))
from test_dp_cpu import ROOT, _port  # noqa: E402


def _parse_lines(text):
    import json

    out = []
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("{"):
            try:
                out.append(json.loads(line))
            except ValueError:
                pass
    return out


def test_rank_exit_is_detected_by_peer():
    """Rank 1 leaves between steps; rank 0's next collective must fail
    within the process-group timeout instead of waiting forever."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", f"--master-port={_port()}", "--max-restarts=0", "-m", "dlvk_b200.parallel.selftest", "--cpu",
           "--mode", "nccl", "--model", "mlp", "--steps", "4", "--fail-rank", "1", "--fail-step", "2",
           "--pg-timeout", "20"]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    t0 = time.monotonic()
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=240, cwd=ROOT, env=env)
    dt = time.monotonic() - t0
    assert r.returncode != 0
    assert dt < 200
    objs = _parse_lines(r.stdout)
    assert any(o.get("injected_exit") == 2 for o in objs), r.stdout[-2000:]


def test_checkpoint_write_failure_keeps_previous_file(tmp_path):
    from dlvk_b200.models.sequential import Sequential

    m = Sequential("cpu", "fp32", seed=0)
    m.add_dense(4, 3)
    m.build()
    path = str(tmp_path / "m.dlvk")
    m.save_weights(path)
    before = open(path, "rb").read()
    os.mkdir(path + ".tmp")  # the writer's temporary file cannot be created
    m.store.master.add_(1.0)
    with pytest.raises(Exception):
        m.save_weights(path)
    assert open(path, "rb").read() == before
    os.rmdir(path + ".tmp")
    # a truncated file is rejected with an exception, not read past its end
    open(str(tmp_path / "t.dlvk"), "wb").write(before[: len(before) // 2])
    m2 = Sequential("cpu", "fp32", seed=0)
    m2.add_dense(4, 3)
    m2.build()
    with pytest.raises(Exception):
        m2.load_weights(str(tmp_path / "t.dlvk"))


def test_error_word_mapping():
    from dlvk_b200.utils import health

    assert health.error_for(0) is None
    assert isinstance(health.error_for(1), health.CommTimeoutError)
    assert isinstance(health.error_for(3), health.PipelineTimeoutError)
    assert type(health.error_for(7)) is health.DeviceError


@pytest.mark.gpu
def test_bounded_peer_wait_times_out_and_context_survives():
    from dlvk_b200 import _ext
    from dlvk_b200.utils import health

    C = _ext.C()
    C.read_device_error(True)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    res = C.comm.wait_flag_probe(flag, 5, 0.3)  # nothing ever writes 5
    torch.cuda.synchronize()
    dt = time.monotonic() - t0
    assert int(res) == 0 and 0.25 < dt < 5.0
    with pytest.raises(health.CommTimeoutError):
        health.check_device()
    # the context is still usable and the error word was cleared
    flag.fill_(5)
    assert int(C.comm.wait_flag_probe(flag, 5, 0.3)) == 1
    y = torch.randn(256, 256, device="cuda").bfloat16()
    C.gemm(y, y)
    health.check_device()


@pytest.mark.gpu
def test_wait_event_deadline():
    from dlvk_b200.utils import health

    ev = torch.cuda.Event()
    ev.record()
    assert health.wait_event(ev, 5.0)
