"""Serve a saved model over HTTP:

    python -m dlvk_b200.deployment.serve model.dlvk [--port 8080] [--max-batch 64]

POST /predict (JSON {"inputs": [...]} or a .dlvk tensor blob), GET /health,
GET /stats."""
from __future__ import annotations

import argparse
import signal
import threading


def main(argv=None):
    from ..models.builder import load_model_file
    from .inference import Config, ModelServingServer

    ap = argparse.ArgumentParser()
    ap.add_argument("model")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-wait-ms", type=float, default=2.0)
    ap.add_argument("--device", default=None)
    a = ap.parse_args(argv)
    model = load_model_file(a.model, a.device)
    cfg = Config()
    cfg.serving.max_batch, cfg.serving.max_wait_ms = a.max_batch, a.max_wait_ms
    srv = ModelServingServer()
    srv.start(model, cfg, a.host, a.port)
    print(f"serving {a.model} on {a.host}:{srv.port}", flush=True)
    done = threading.Event()
    signal.signal(signal.SIGTERM, lambda *_: done.set())
    signal.signal(signal.SIGINT, lambda *_: done.set())
    done.wait()
    srv.stop()


if __name__ == "__main__":
    main()
