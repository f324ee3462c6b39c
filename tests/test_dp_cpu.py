"""Data-parallel host logic (bucketing, gradient hooks, per-bucket reduce +
optimizer, shard consolidation) with 2 gloo ranks on CPU, against
single-process full-batch training."""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run_selftest(nproc, extra, timeout=240):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr", "127.0.0.1", f"--master-port={_port()}", "-m", "dlvk_b200.parallel.selftest"] + extra
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=ROOT, env=env)
    return r.returncode, parse_objects(r.stdout), r.stdout + r.stderr


def parse_objects(text):
    """Every JSON object in `text` that carries an "ok" key (rank outputs
    can interleave on the shared pipe, so lines are not trusted)."""
    dec, out, i = json.JSONDecoder(), [], 0
    while True:
        i = text.find("{", i)
        if i < 0:
            return out
        try:
            obj, end = dec.raw_decode(text, i)
        except json.JSONDecodeError:
            i += 1
            continue
        if isinstance(obj, dict) and "ok" in obj:
            out.append(obj)
        i = end


@pytest.mark.parametrize("model", ["mlp", "transformer"])
def test_dp_gloo_matches_full_batch(model):
    rc, lines, log = run_selftest(2, ["--cpu", "--mode", "nccl", "--model", model])
    assert rc == 0, log[-3000:]
    assert len(lines) == 2 and all(l["ok"] for l in lines), lines
