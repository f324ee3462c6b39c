"""Python side of the `.dlvk` model format (the byte layout is implemented in
C++, csrc/runtime/dlvk_io.cpp).

A v2 file holds every model tensor (fp32 master weights and batch-norm
running statistics), optionally the optimizer state (m / v / momentum
buffers plus step and hyper-parameters in the metadata) and the RNG state
(seed and device step counter), so a resumed run continues bit-exactly.
Metadata JSON is written with sorted keys and no clock values, so saving,
loading and saving again reproduces the same bytes.
"""
from __future__ import annotations

import json
from typing import Optional

import torch

from .. import _ext

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.int32: 3, torch.int8: 4,
               torch.uint8: 5, torch.int64: 6}
CODE_DTYPES = {v: k for k, v in DTYPE_CODES.items()}


def tensor_record(name: str, t: torch.Tensor):
    c = t.detach().contiguous().cpu()
    raw = c.view(torch.uint8).numpy().tobytes() if c.numel() else b""
    return (name, DTYPE_CODES[c.dtype], list(c.shape), raw)


def record_tensor(rec) -> torch.Tensor:
    name, code, dims, raw = rec
    dt = CODE_DTYPES[int(code)]
    if len(raw) == 0:
        return torch.empty(dims, dtype=dt)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dt).reshape(dims).clone()


def save(path: str, meta: dict, tensors) -> None:
    _ext.C().io.save_v2(path, json.dumps(meta, sort_keys=True, separators=(",", ":")),
                        [tensor_record(n, t) for n, t in tensors])


def encode(meta: dict, tensors) -> bytes:
    return _ext.C().io.encode_v2(json.dumps(meta, sort_keys=True, separators=(",", ":")),
                                 [tensor_record(n, t) for n, t in tensors])


def load(path: str):
    """Returns (version, variant, meta dict, {name: tensor})."""
    version, variant, meta_json, recs = _ext.C().io.load(path)
    try:
        meta = json.loads(meta_json) if meta_json else {}
    except json.JSONDecodeError:
        meta = {"raw": meta_json}
    return version, variant, meta, {r[0]: record_tensor(r) for r in recs}


def save_model(path: str, model, optimizer=None, extra_meta: Optional[dict] = None) -> None:
    model.build()
    tensors = list(model.state_tensors())
    meta = {"framework": "dlvk_b200", "format_version": 2, "architecture": model.architecture(),
            "compute_dtype": str(model.dtype).replace("torch.", ""),
            "rng": {"seed": int(model.dev.seed), "step": int(model.dev.step_t.item())}}
    if optimizer is not None:
        meta["optimizer"] = optimizer.state_meta(model.store)
        tensors += list(optimizer.state_tensors(model.store))
    if extra_meta:
        meta["extra"] = extra_meta
    save(path, meta, tensors)


def load_model(path: str, model, optimizer=None) -> dict:
    version, variant, meta, tens = load(path)
    model.build()
    if variant == "v1-weights":
        _load_v1_weights(model, tens)
        return meta
    if variant == "v1-header":
        return meta  # the reference's header-only files carry no tensors
    for name, t in model.state_tensors():
        if name not in tens:
            raise KeyError(f".dlvk file has no tensor '{name}'")
        src = tens[name]
        if tuple(src.shape) != tuple(t.shape):
            raise ValueError(f"{name}: shape {tuple(src.shape)} in file, {tuple(t.shape)} in model")
        t.copy_(src.to(t.device, t.dtype))
    model.store.sync_value()
    rng = meta.get("rng")
    if rng:
        model.dev.seed = int(rng.get("seed", model.dev.seed))
        model.dev.step_t.fill_(int(rng.get("step", 0)))
    if optimizer is not None and "optimizer" in meta:
        for name, t in optimizer.state_tensors(model.store):
            if name in tens:
                t.copy_(tens[name].to(t.device, t.dtype))
        optimizer.load_state_meta(model.store, meta["optimizer"])
    return meta


def _load_v1_weights(model, tens) -> None:
    """The reference's weight-bearing v1 sample stores one dense layer's
    flattened weights and biases."""
    from ..models.layers import DenseLayer

    dense = [l for l in model.m_layers if isinstance(l, DenseLayer)]
    if not dense:
        raise ValueError("v1 weight file needs a model with a Dense layer")
    d = dense[0]
    w, b = tens["weights"], tens["biases"]
    d.weight.master.copy_(w.reshape(d.weight.shape).to(d.weight.master.device))
    if d.bias is not None:
        d.bias.master.copy_(b.reshape(d.bias.shape).to(d.bias.master.device))
    model.store.sync_value()


def decode(blob: bytes):
    """Like `load` for an in-memory `.dlvk` blob."""
    version, variant, meta_json, recs = _ext.C().io.decode(blob)
    try:
        meta = json.loads(meta_json) if meta_json else {}
    except json.JSONDecodeError:
        meta = {"raw": meta_json}
    return version, variant, meta, {r[0]: record_tensor(r) for r in recs}
