"""Data-parallel recovery: a 2-rank gloo job trains 3 steps, checkpoints
and stops; a new job loads the checkpoint and trains 2 more steps.  The
final `.dlvk` (weights, Adam state, step counters) must equal, byte for
byte, that of 5 uninterrupted steps (dlvk_b200/deployment/
recovery_selftest.py)."""
import os
import subprocess
import sys

from test_dp_cpu import ROOT, _port, parse_objects


def _phase(phase, d):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", f"--master-port={_port()}", "--max-restarts=0", "-m", "dlvk_b200.deployment.recovery_selftest",
           "--phase", phase, "--dir", str(d), "--cpu"]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    objs = parse_objects(r.stdout)
    assert len(objs) == 2 and all(o["ok"] for o in objs), objs


def test_restart_from_checkpoint_is_bit_identical(tmp_path):
    _phase("full", tmp_path)
    _phase("first", tmp_path)
    _phase("resume", tmp_path)
    full = (tmp_path / "full.dlvk").read_bytes()
    resumed = (tmp_path / "resumed.dlvk").read_bytes()
    ckpt = (tmp_path / "ckpt.dlvk").read_bytes()
    assert ckpt != full  # the checkpoint is the 3-step state
    assert resumed == full
