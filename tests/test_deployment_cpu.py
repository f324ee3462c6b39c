"""Deployment on CPU: dynamic-batching engine, HTTP server, packaging,
container manifests, and the multi-GPU trainer API on 2 gloo ranks."""
import json
import os
import subprocess
import sys
import urllib.request

import torch

from dlvk_b200.deployment import (CrossPlatformDeployment, DeviceConstraints, EdgeDeploymentOptimizer,
                                  ModelInferenceEngine, ModelServingServer, deserialize_tensors, serialize_tensors)
from dlvk_b200.models.sequential import Sequential

sys.path.insert(0, os.path.dirname(__file__))
from test_dp_cpu import ROOT, _port, parse_objects  # noqa: E402


def model():
    m = Sequential("cpu", "fp32", seed=0)
    m.add_dense(8, 16).add_relu().add_dense(16, 3).add_softmax()
    m.build()
    m.set_training(False)
    return m


def test_engine_batches_requests():
    m = model()
    eng = ModelInferenceEngine(m)
    eng.config.serving.max_wait_ms = 20.0
    xs = [torch.randn(1, 8) for _ in range(40)]
    outs = [f.result(10) for f in [eng.infer_async(x) for x in xs]]
    assert torch.allclose(torch.cat(outs), m.forward(torch.cat(xs)), atol=1e-6)
    st = eng.stats()
    assert st["requests_samples"] == 40 and st["batches"] < 40
    got = []
    eng.infer_async(xs[0], callback=lambda o: got.append(o[0])).result(10)
    assert len(got) == 1
    eng.finalize()


def test_http_server_json_and_binary():
    m = model()
    srv = ModelServingServer()
    srv.start(m)
    try:
        x = torch.randn(3, 8)
        req = urllib.request.Request(srv.url() + "/predict", data=json.dumps({"inputs": x.tolist()}).encode(),
                                     headers={"Content-Type": "application/json"})
        out = torch.tensor(json.loads(urllib.request.urlopen(req).read())["outputs"])
        assert torch.allclose(out, m.forward(x), atol=1e-6)
        req = urllib.request.Request(srv.url() + "/predict", data=serialize_tensors([x]),
                                     headers={"Content-Type": "application/octet-stream"})
        y = deserialize_tensors(urllib.request.urlopen(req).read())[0]
        assert torch.allclose(y, m.forward(x), atol=1e-6)
        assert json.loads(urllib.request.urlopen(srv.url() + "/health").read())["status"] == "ok"
        assert json.loads(urllib.request.urlopen(srv.url() + "/stats").read())["requests_samples"] == 6
    finally:
        srv.stop()


def test_packaging_and_manifests(tmp_path):
    m = model()
    assert EdgeDeploymentOptimizer.generate_deployment_package(m, str(tmp_path / "pkg"), "cuda", input_shape=[1, 8])
    man = json.loads((tmp_path / "pkg" / "manifest.json").read_text())
    assert set(man["files"]) == {"dlvk", "safetensors", "onnx"} and man["parameters"] == m.parameter_count()
    assert CrossPlatformDeployment.create_docker_container(m, "dlvk/mlp:1", ["A=1"], str(tmp_path / "d"))
    assert "ENV A=1" in (tmp_path / "d" / "Dockerfile").read_text()
    assert CrossPlatformDeployment.create_kubernetes_deployment(m, "mlp", 3, str(tmp_path))
    assert "replicas: 3" in (tmp_path / "mlp.yaml").read_text()
    small = EdgeDeploymentOptimizer.apply_memory_optimizations(m, DeviceConstraints(max_memory_bytes=300))
    assert float((small.store.master == 0).float().mean()) > 0.5
    assert EdgeDeploymentOptimizer.estimate_model_latency(m) > 0


def test_multi_gpu_trainer_gloo():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", f"--master-port={_port()}", "-m", "dlvk_b200.deployment.selftest", "--cpu"]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT, env=env)
    res = parse_objects(r.stdout)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert len(res) == 2 and all(o["ok"] for o in res), res
