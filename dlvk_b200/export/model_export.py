"""Model export manager (include/dlvk/export/model_export.h:25-253,
src/export/model_export.cpp).

Formats and what is written:

* DLVK: the `.dlvk` v2 container (native C++ writer) with every weight,
  the architecture and optional optimizer state.
* ONNX: a binary ModelProto, opset 17 (export/onnx.py).
* GGUF: GGUF v3 (native C++), tensors in their stored dtype, metadata
  keys `general.architecture = "dlvk"`, `general.name`, `dlvk.architecture`
  (JSON) and the reference's size fields (`dlvk.vocab_size`, ...).
* SafeTensors: native C++ writer; `__metadata__` carries the architecture.
* HDF5: needs h5py, which this image does not have; `export_model` raises
  a clear error for it (the reference compiled it only with
  DLVK_HDF5_SUPPORT, src/export/format_specific.cpp:16-219).

The reference's exporters wrote no tensor data (`extract_tensors` returned
an empty list, model_export.cpp:17-48); here every format round-trips the
weights, and `import_model` rebuilds the Sequential from the stored
architecture.
"""
from __future__ import annotations

import enum
import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from .. import _ext

_DTYPE_NAMES = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16", torch.int32: "I32",
                torch.int8: "I8", torch.uint8: "U8", torch.int64: "I64", torch.float64: "F64"}
_NAME_DTYPES = {v: k for k, v in _DTYPE_NAMES.items()}


class ModelFormat(enum.Enum):
    DLVK = 0
    ONNX = 1
    GGUF = 2
    HDF5 = 3
    SAFETENSORS = 4
    TENSORFLOW_SAVEDMODEL = 5


@dataclass
class ModelMetadata:
    name: str = "dlvk_model"
    architecture: str = "sequential"
    version: str = "1.0"
    framework: str = "dlvk_b200"
    custom_metadata: Dict[str, str] = field(default_factory=dict)
    vocab_size: int = 0
    embedding_dim: int = 0
    hidden_size: int = 0
    sequence_length: int = 0
    num_layers: int = 0


@dataclass
class TensorInfo:
    name: str
    shape: List[int]
    dtype: torch.dtype
    data: torch.Tensor
    offset: int = 0
    size_bytes: int = 0


def extract_tensors(model) -> List[TensorInfo]:
    model.build()
    out, off = [], 0
    for name, t in model.state_tensors():
        c = t.detach().cpu().contiguous()
        nb = c.numel() * c.element_size()
        out.append(TensorInfo(name, list(c.shape), c.dtype, c, off, nb))
        off += nb
    return out


def _raw(t: torch.Tensor) -> bytes:
    return t.contiguous().view(torch.uint8).numpy().tobytes() if t.numel() else b""


def _from_raw(raw: bytes, dtype: torch.dtype, shape) -> torch.Tensor:
    if not raw:
        return torch.empty(shape, dtype=dtype)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dtype).reshape(shape).clone()


def _load_into(model, tensors: Dict[str, torch.Tensor]) -> None:
    for name, t in model.state_tensors():
        if name not in tensors:
            raise KeyError(f"imported file has no tensor '{name}'")
        t.copy_(tensors[name].reshape(t.shape).to(t.device, t.dtype))
    model.store.sync_value()


def _rebuild(arch_json: str, device=None, dtype="fp32"):
    from ..models.builder import model_from_architecture

    return model_from_architecture(json.loads(arch_json), device, dtype)


class ModelExporter:
    format = None

    def export_model(self, model, filename: str, metadata: ModelMetadata) -> bool:
        raise NotImplementedError

    def import_model(self, filename: str, device=None) -> Tuple[object, ModelMetadata]:
        raise NotImplementedError

    def extract_tensors(self, model) -> List[TensorInfo]:
        return extract_tensors(model)


def _meta_dict(model, md: ModelMetadata) -> Dict[str, str]:
    d = {"name": md.name, "architecture": md.architecture, "version": md.version, "framework": md.framework,
         "dlvk.architecture": json.dumps(model.architecture())}
    for k in ("vocab_size", "embedding_dim", "hidden_size", "sequence_length", "num_layers"):
        d[k] = str(getattr(md, k))
    d.update({str(k): str(v) for k, v in md.custom_metadata.items()})
    return d


def _md_from(d: Dict[str, str]) -> ModelMetadata:
    md = ModelMetadata()
    for k in ("name", "architecture", "version", "framework"):
        if k in d:
            setattr(md, k, d[k])
    for k in ("vocab_size", "embedding_dim", "hidden_size", "sequence_length", "num_layers"):
        if k in d:
            try:
                setattr(md, k, int(d[k]))
            except ValueError:
                pass
    known = {"name", "architecture", "version", "framework", "dlvk.architecture", "vocab_size", "embedding_dim",
             "hidden_size", "sequence_length", "num_layers"}
    md.custom_metadata = {k: v for k, v in d.items() if k not in known}
    return md


class DLVKExporter(ModelExporter):
    format = ModelFormat.DLVK

    def export_model(self, model, filename, metadata):
        from ..utils import dlvk_io

        dlvk_io.save_model(filename, model, extra_meta={"export_metadata": metadata.__dict__})
        return True

    def import_model(self, filename, device=None):
        from ..models.builder import load_model_file
        from ..utils import dlvk_io

        m = load_model_file(filename, device)
        _, _, meta, _ = dlvk_io.load(filename)
        em = (meta.get("extra") or {}).get("export_metadata") or {}
        md = ModelMetadata(**{k: v for k, v in em.items() if k in ModelMetadata.__dataclass_fields__})
        return m, md


class SafeTensorsExporter(ModelExporter):
    format = ModelFormat.SAFETENSORS

    def export_model(self, model, filename, metadata):
        recs = [(t.name, _DTYPE_NAMES[t.dtype], t.shape, _raw(t.data)) for t in extract_tensors(model)]
        meta = sorted(_meta_dict(model, metadata).items())
        blob = _ext.C().export.encode_safetensors(recs, meta)
        _atomic_write(filename, blob)
        return True

    def import_model(self, filename, device=None):
        with open(filename, "rb") as f:
            recs, meta = _ext.C().export.decode_safetensors(f.read())
        meta = dict(meta)
        if "dlvk.architecture" not in meta:
            raise ValueError(f"{filename}: no dlvk.architecture in __metadata__")
        m = _rebuild(meta["dlvk.architecture"], device)
        _load_into(m, {n: _from_raw(raw, _NAME_DTYPES[dt], shape) for n, dt, shape, raw in recs})
        return m, _md_from(meta)


class GGUFExporter(ModelExporter):
    format = ModelFormat.GGUF
    alignment = 32

    def export_model(self, model, filename, metadata):
        recs = [(t.name, _DTYPE_NAMES[t.dtype], t.shape, _raw(t.data)) for t in extract_tensors(model)]
        md = _meta_dict(model, metadata)
        kvs = [("general.architecture", 8, "dlvk"), ("general.name", 8, metadata.name),
               ("general.version", 8, metadata.version), ("dlvk.architecture", 8, md["dlvk.architecture"])]
        for k in ("vocab_size", "embedding_dim", "hidden_size", "sequence_length", "num_layers"):
            kvs.append((f"dlvk.{k}", 4, int(getattr(metadata, k))))
        for k, v in metadata.custom_metadata.items():
            kvs.append((f"dlvk.custom.{k}", 8, str(v)))
        blob = _ext.C().export.encode_gguf(recs, kvs, self.alignment)
        _atomic_write(filename, blob)
        return True

    def import_model(self, filename, device=None):
        with open(filename, "rb") as f:
            recs, kvs = _ext.C().export.decode_gguf(f.read())
        kv = {k: v for k, _, v in kvs}
        if "dlvk.architecture" not in kv:
            raise ValueError(f"{filename}: not a dlvk GGUF file (no dlvk.architecture)")
        m = _rebuild(kv["dlvk.architecture"], device)
        _load_into(m, {n: _from_raw(raw, _NAME_DTYPES[dt], shape) for n, dt, shape, raw in recs})
        d = {"name": kv.get("general.name", ""), "version": kv.get("general.version", "")}
        for k in ("vocab_size", "embedding_dim", "hidden_size", "sequence_length", "num_layers"):
            if f"dlvk.{k}" in kv:
                d[k] = str(kv[f"dlvk.{k}"])
        d.update({k[len("dlvk.custom."):]: str(v) for k, v in kv.items() if k.startswith("dlvk.custom.")})
        return m, _md_from(d)


class ONNXExporter(ModelExporter):
    format = ModelFormat.ONNX

    def __init__(self, input_shape: Optional[List[int]] = None):
        self.input_shape = input_shape

    def export_model(self, model, filename, metadata, input_shape=None):
        from . import onnx

        shape = input_shape or self.input_shape or _guess_input_shape(model)
        onnx.export_model(model, filename, shape, {k: v for k, v in _meta_dict(model, metadata).items()
                                                   if k != "dlvk.architecture"})
        return True

    def import_model(self, filename, device=None):
        from . import onnx

        with open(filename, "rb") as f:
            parsed = onnx.parse_model(f.read())
        meta = parsed["metadata"]
        m = _rebuild(meta["dlvk.architecture"], device)
        _load_onnx_weights(m, parsed)
        return m, _md_from(meta)


class HDF5Exporter(ModelExporter):
    format = ModelFormat.HDF5

    def _h5py(self):
        try:
            import h5py  # noqa: F401

            return h5py
        except ImportError as e:
            raise RuntimeError("HDF5 export needs the h5py package, which is not installed") from e

    def export_model(self, model, filename, metadata):
        h5py = self._h5py()
        with h5py.File(filename, "w") as f:
            for k, v in _meta_dict(model, metadata).items():
                f.attrs[k] = v
            g = f.create_group("weights")
            for t in extract_tensors(model):
                g.create_dataset(t.name, data=t.data.float().numpy())
        return True

    def import_model(self, filename, device=None):
        h5py = self._h5py()
        with h5py.File(filename, "r") as f:
            meta = {k: str(v) for k, v in f.attrs.items()}
            m = _rebuild(meta["dlvk.architecture"], device)
            _load_into(m, {k: torch.from_numpy(f["weights"][k][()]) for k in f["weights"]})
        return m, _md_from(meta)


def _guess_input_shape(model) -> List[int]:
    from ..models import layers as L

    first = model.m_layers[0]
    if isinstance(first, L.DenseLayer):
        return [1, first.input_size]
    if isinstance(first, L.Conv2DLayer):
        raise ValueError("pass input_shape=[N, C, H, W] to export a convolutional model to ONNX")
    if isinstance(first, (L.EmbeddingLayer, L.PositionalEncodingLayer, L.TransformerEncoderLayer)):
        raise ValueError("pass input_shape=[N, S(, D)] to export a sequence model to ONNX")
    raise ValueError("pass input_shape to export this model to ONNX")


def _load_onnx_weights(model, parsed) -> None:
    """Initializers named `param.<i>` are the model's i-th parameter,
    `buf.<layer>.mean|var` BatchNorm running statistics and
    `rec.<layer>.W|R|B` the ONNX-ordered recurrent stacks."""
    from ..models import layers as L

    inits = parsed["initializers"]
    params = model.parameters()
    seen = set()
    for name, t in inits.items():
        if name.startswith("param."):
            p = params[int(name.split(".")[1])]
            p.master.copy_(t.reshape(p.shape).to(p.master.device, torch.float32))
            seen.add(id(p))
        elif name.startswith("buf."):
            _, li, kind = name.split(".")
            layer = model.m_layers[int(li)]
            getattr(layer, "running_" + kind).copy_(t.to(layer.running_mean.device))
    for li, layer in enumerate(model.m_layers):
        if isinstance(layer, (L.RNNLayer, L.LSTMLayer, L.GRULayer, L.BidirectionalRNN)):
            cells = [layer.fwd, layer.bwd] if isinstance(layer, L.BidirectionalRNN) else [layer]
            W, R, B = (inits[f"rec.{li}.{k}"] for k in ("W", "R", "B"))
            H, kind = cells[0].hidden_size, cells[0].kind
            inv = {1: [0, 2, 3, 1], 2: [1, 0, 2], 0: [0]}[kind]  # ONNX gate order -> ours
            G = len(inv)

            def back(t):
                parts = t.reshape(G, H, *t.shape[1:])
                return torch.cat([parts[j] for j in inv], 0)

            for d, c in enumerate(cells):
                for p, v in ((c.w_ih, back(W[d])), (c.w_hh, back(R[d]))):
                    p.master.copy_(v.to(p.master.device))
                    seen.add(id(p))
                if c.b_ih is not None:
                    for p, v in ((c.b_ih, back(B[d][:G * H])), (c.b_hh, back(B[d][G * H:]))):
                        p.master.copy_(v.to(p.master.device))
                        seen.add(id(p))
    missing = [p.name for p in params if id(p) not in seen]
    if missing:
        raise ValueError(f"ONNX file lacks parameters {missing[:4]}...")
    model.store.sync_value()


def _atomic_write(path: str, blob: bytes) -> None:
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(blob)
    os.replace(tmp, path)


class ModelExportManager:
    _EXT = {ModelFormat.DLVK: ".dlvk", ModelFormat.ONNX: ".onnx", ModelFormat.GGUF: ".gguf",
            ModelFormat.HDF5: ".h5", ModelFormat.SAFETENSORS: ".safetensors",
            ModelFormat.TENSORFLOW_SAVEDMODEL: ".savedmodel"}

    def __init__(self):
        self.exporters = {ModelFormat.DLVK: DLVKExporter(), ModelFormat.ONNX: ONNXExporter(),
                          ModelFormat.GGUF: GGUFExporter(), ModelFormat.SAFETENSORS: SafeTensorsExporter(),
                          ModelFormat.HDF5: HDF5Exporter()}

    def export_model(self, model, filename: str, format: ModelFormat, metadata: Optional[ModelMetadata] = None,
                     **kw) -> bool:
        ex = self.exporters.get(format)
        if ex is None:
            raise NotImplementedError(f"no exporter for {format.name}")
        return ex.export_model(model, filename, metadata or ModelMetadata(), **kw)

    def import_model(self, filename: str, format: Optional[ModelFormat] = None, device=None):
        fmt = format or self.detect_format(filename)
        ex = self.exporters.get(fmt)
        if ex is None:
            raise NotImplementedError(f"no importer for {fmt.name}")
        return ex.import_model(filename, device)

    def detect_format(self, filename: str) -> ModelFormat:
        low = filename.lower()
        for fmt, ext in self._EXT.items():
            if low.endswith(ext):
                return fmt
        if low.endswith(".hdf5"):
            return ModelFormat.HDF5
        return ModelFormat.DLVK

    def export_all_formats(self, model, base_filename: str, metadata: Optional[ModelMetadata] = None,
                           input_shape=None) -> bool:
        ok = True
        for fmt in self.get_supported_formats():
            kw = {"input_shape": input_shape} if fmt is ModelFormat.ONNX else {}
            try:
                ok &= self.export_model(model, base_filename + self._EXT[fmt], fmt, metadata, **kw)
            except (RuntimeError, ValueError, NotImplementedError):
                ok = False
        return ok

    def get_supported_formats(self) -> List[ModelFormat]:
        fmts = [ModelFormat.DLVK, ModelFormat.ONNX, ModelFormat.GGUF, ModelFormat.SAFETENSORS]
        try:
            import h5py  # noqa: F401

            fmts.append(ModelFormat.HDF5)
        except ImportError:
            pass
        return fmts

    def get_extension(self, format: ModelFormat) -> str:
        return self._EXT[format]


def create_export_manager() -> ModelExportManager:
    return ModelExportManager()
