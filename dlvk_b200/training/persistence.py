"""Model persistence (include/dlvk/training/model_persistence.h:17-383,
src/training/model_persistence.cpp).

* `ModelSerializer`: `.dlvk` binary (v2 container with every weight,
  the architecture, optimizer state and RNG) and a JSON form
  (architecture + metadata + weights as nested lists); `load_*` rebuild
  the model (the reference wrote header-only files with
  param_count = 0 and `load_binary` returned nullptr,
  model_persistence.cpp:13-124).
* `ModelCheckpoint` (checkpoint manager): `{dir}/{name}_epoch_{%04d}.dlvk`
  plus `{dir}/{name}_metrics_{%04d}.json`, best-only / every
  `save_frequency` epochs, keeps at most `max_checkpoints` (oldest
  deleted), tracks the best checkpoint (model_persistence.cpp:149-221).
* `ModelVersioning`: `{experiment_dir}/{experiment}/v%03d/model.dlvk` +
  `version_info.json`, list / load / compare versions
  (model_persistence.cpp:224-282; directories are created with
  os.makedirs instead of `system("mkdir -p")`).
* `CheckpointData` gathers what a resume needs: weights, optimizer state,
  epoch / step / lr, metrics history and the Philox RNG seed / counter.
"""
from __future__ import annotations

import enum
import glob
import json
import os
import time
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

import torch

from .callbacks import TrainingCallback, TrainingMetrics


class SerializationFormat(enum.Enum):
    DLVK_BINARY = 0
    DLVK_JSON = 1
    HDF5 = 2
    ONNX = 3
    NUMPY_NPZ = 4


@dataclass
class ModelMetadata:
    name: str = ""
    description: str = ""
    version: str = "1.0"
    framework_version: str = "dlvk_b200"
    custom_fields: Dict[str, str] = field(default_factory=dict)

    @property
    def model_name(self) -> str:
        return self.name


@dataclass
class CheckpointData:
    metadata: ModelMetadata = field(default_factory=ModelMetadata)
    weights: Dict[str, torch.Tensor] = field(default_factory=dict)
    optimizer_state: Dict[str, torch.Tensor] = field(default_factory=dict)
    optimizer_params: Dict[str, float] = field(default_factory=dict)
    current_epoch: int = 0
    current_step: int = 0
    current_lr: float = 0.0
    current_metrics: Optional[TrainingMetrics] = None
    training_history: List[TrainingMetrics] = field(default_factory=list)
    random_seed: int = 0
    rng_state: List[int] = field(default_factory=list)


def _metrics_from(d: dict) -> TrainingMetrics:
    m = TrainingMetrics()
    for k, v in d.items():
        key = {"val_loss": "validation_loss", "val_accuracy": "validation_accuracy"}.get(k, k)
        if hasattr(m, key) and not isinstance(getattr(type(m), key, None), property):
            setattr(m, key, type(getattr(m, key))(v))
    return m


class ModelSerializer:
    def __init__(self, fmt: SerializationFormat = SerializationFormat.DLVK_BINARY):
        self.format = fmt

    # binary .dlvk
    def save_binary(self, model, filepath: str, metadata: Optional[ModelMetadata] = None, optimizer=None,
                    extra: Optional[dict] = None) -> bool:
        em = {"metadata": asdict(metadata or ModelMetadata())}
        if extra:
            em.update(extra)
        model.save_weights(filepath, optimizer=optimizer, extra_meta=em)
        return True

    def load_binary(self, filepath: str, device=None, optimizer=None):
        from ..models.builder import load_model_file

        return load_model_file(filepath, device, optimizer=optimizer)

    # JSON
    def save_json(self, model, filepath: str, metadata: Optional[ModelMetadata] = None) -> bool:
        model.build()
        doc = {"format": "dlvk-json", "version": 2, "metadata": asdict(metadata or ModelMetadata()),
               "architecture": model.architecture(), "compute_dtype": str(model.dtype).replace("torch.", ""),
               "weights": {n: {"shape": list(t.shape), "data": t.detach().float().cpu().reshape(-1).tolist()}
                           for n, t in model.state_tensors()}}
        tmp = filepath + ".tmp"
        with open(tmp, "w") as f:
            json.dump(doc, f)
        os.replace(tmp, filepath)
        return True

    def load_json(self, filepath: str, device=None):
        from ..models.builder import model_from_architecture

        with open(filepath) as f:
            doc = json.load(f)
        m = model_from_architecture(doc["architecture"], device, doc.get("compute_dtype", "float32"))
        w = doc["weights"]
        for n, t in m.state_tensors():
            t.copy_(torch.tensor(w[n]["data"], dtype=torch.float32).reshape(t.shape).to(t.device, t.dtype))
        m.store.sync_value()
        return m

    def save(self, model, filepath: str, metadata: Optional[ModelMetadata] = None) -> bool:
        if self.format is SerializationFormat.DLVK_JSON:
            return self.save_json(model, filepath, metadata)
        if self.format is SerializationFormat.ONNX:
            from ..export import ModelExportManager, ModelFormat

            return ModelExportManager().export_model(model, filepath, ModelFormat.ONNX)
        if self.format is SerializationFormat.HDF5:
            from ..export import ModelExportManager, ModelFormat

            return ModelExportManager().export_model(model, filepath, ModelFormat.HDF5)
        if self.format is SerializationFormat.NUMPY_NPZ:
            return self.export_to_numpy(model, filepath)
        return self.save_binary(model, filepath, metadata)

    def load(self, filepath: str, device=None):
        if self.format is SerializationFormat.DLVK_JSON:
            return self.load_json(filepath, device)
        return self.load_binary(filepath, device)

    @staticmethod
    def serialize_metadata(metadata: ModelMetadata) -> str:
        return json.dumps(asdict(metadata))

    # Static entry points of include/dlvk/training/model_persistence.h:203-239.
    @staticmethod
    def save_model(model, filepath: str, format: SerializationFormat = SerializationFormat.DLVK_BINARY,
                   metadata: Optional[ModelMetadata] = None) -> bool:
        return ModelSerializer(format).save(model, filepath, metadata)

    @staticmethod
    def load_model(filepath: str, format: SerializationFormat = SerializationFormat.DLVK_BINARY, device=None):
        return ModelSerializer(format).load(filepath, device)

    @staticmethod
    def save_weights(model, filepath: str, format: SerializationFormat = SerializationFormat.DLVK_BINARY) -> bool:
        """Weights only, into an existing architecture's layout: `.dlvk`
        binary, JSON (the same document save_json writes) or NumPy `.npz`."""
        if format is SerializationFormat.NUMPY_NPZ:
            return ModelSerializer.export_to_numpy(model, filepath)
        if format is SerializationFormat.DLVK_JSON:
            return ModelSerializer(format).save_json(model, filepath)
        if format is not SerializationFormat.DLVK_BINARY:
            raise ValueError(f"save_weights supports DLVK_BINARY, DLVK_JSON and NUMPY_NPZ, not {format.name}")
        model.save_weights(filepath)
        return True

    @staticmethod
    def load_weights(model, filepath: str, format: SerializationFormat = SerializationFormat.DLVK_BINARY) -> bool:
        """Loads weights written by save_weights into `model` (same layer
        list); every tensor's shape must match."""
        model.build()
        if format is SerializationFormat.DLVK_BINARY:
            model.load_weights(filepath)
            return True
        if format is SerializationFormat.DLVK_JSON:
            with open(filepath) as f:
                w = json.load(f)["weights"]
            src = {n: torch.tensor(e["data"], dtype=torch.float32).reshape(e["shape"]) for n, e in w.items()}
        elif format is SerializationFormat.NUMPY_NPZ:
            import numpy as np

            with np.load(filepath) as z:
                src = {n: torch.from_numpy(z[n].astype("float32")) for n in z.files}
        else:
            raise ValueError(f"load_weights supports DLVK_BINARY, DLVK_JSON and NUMPY_NPZ, not {format.name}")
        for n, t in model.state_tensors():
            if n not in src:
                raise ValueError(f"{filepath}: no tensor named {n}")
            if tuple(src[n].shape) != tuple(t.shape):
                raise ValueError(f"{filepath}: {n} has shape {tuple(src[n].shape)}, the model {tuple(t.shape)}")
            t.copy_(src[n].to(t.device, t.dtype))
        model.store.sync_value()
        return True

    @staticmethod
    def export_to_onnx(model, filepath: str, input_shapes=None) -> bool:
        """ONNX graph with the weights as initializers; `input_shapes` is a
        list with one input shape (the model has one input)."""
        from ..export import ModelExportManager, ModelFormat

        shape = list(input_shapes[0]) if input_shapes else None
        return ModelExportManager().export_model(model, filepath, ModelFormat.ONNX, input_shape=shape)

    @staticmethod
    def export_to_numpy(model, filepath: str) -> bool:
        """Every parameter and buffer as an fp32 array in one `.npz`, keyed
        by the names state_tensors() gives."""
        import numpy as np

        model.build()
        tmp = filepath + ".tmp.npz"
        np.savez(tmp, **{n: t.detach().float().cpu().numpy() for n, t in model.state_tensors()})
        os.replace(tmp, filepath)
        return True

    # CheckpointData <-> file
    @staticmethod
    def save_checkpoint_data(data: CheckpointData, filepath: str, model, optimizer=None) -> bool:
        extra = {"checkpoint": {"epoch": data.current_epoch, "step": data.current_step, "lr": data.current_lr,
                                "metrics": data.current_metrics.as_dict() if data.current_metrics else None,
                                "history": [h.as_dict() for h in data.training_history],
                                "optimizer_params": data.optimizer_params},
                 "metadata": asdict(data.metadata)}
        model.save_weights(filepath, optimizer=optimizer, extra_meta=extra)
        return True

    @staticmethod
    def load_checkpoint_data(filepath: str, model=None, optimizer=None) -> CheckpointData:
        from ..utils import dlvk_io

        _, _, meta, tens = dlvk_io.load(filepath)
        ex = (meta.get("extra") or {})
        ck = ex.get("checkpoint") or {}
        data = CheckpointData(metadata=ModelMetadata(**ex.get("metadata", {})) if ex.get("metadata") else
                              ModelMetadata())
        data.weights = {k: v for k, v in tens.items() if not k.startswith("optim.")}
        data.optimizer_state = {k: v for k, v in tens.items() if k.startswith("optim.")}
        data.current_epoch = int(ck.get("epoch", 0))
        data.current_step = int(ck.get("step", 0))
        data.current_lr = float(ck.get("lr", 0.0))
        data.current_metrics = _metrics_from(ck["metrics"]) if ck.get("metrics") else None
        data.training_history = [_metrics_from(h) for h in ck.get("history", [])]
        data.optimizer_params = ck.get("optimizer_params", {})
        rng = meta.get("rng") or {}
        data.random_seed = int(rng.get("seed", 0))
        data.rng_state = [int(rng.get("step", 0))]
        if model is not None:
            model.load_weights(filepath, optimizer=optimizer)
        return data


class ModelCheckpoint:
    """Checkpoint manager (the training-namespace class; the Keras-style
    callback of the same name lives in training.callbacks)."""

    def __init__(self, checkpoint_dir: str, model_name: str = "model",
                 format: SerializationFormat = SerializationFormat.DLVK_BINARY, save_best_only: bool = True,
                 monitor_metric: str = "val_loss", maximize_metric: bool = False, save_frequency: int = 1,
                 max_checkpoints: int = 5):
        self.checkpoint_dir = checkpoint_dir
        self.model_name = model_name
        self.format = format
        self.save_best_only = save_best_only
        self.monitor_metric = monitor_metric
        self.maximize_metric = maximize_metric
        self.save_frequency = max(1, int(save_frequency))
        self.max_checkpoints = int(max_checkpoints)
        self.best_metric_value = -float("inf") if maximize_metric else float("inf")
        self.best_checkpoint_path = ""
        self.checkpoint_history: List[str] = []
        os.makedirs(checkpoint_dir, exist_ok=True)

    def generate_checkpoint_filename(self, epoch: int, metric_value: float = 0.0) -> str:
        ext = ".json" if self.format is SerializationFormat.DLVK_JSON else ".dlvk"
        return os.path.join(self.checkpoint_dir, f"{self.model_name}_epoch_{epoch:04d}{ext}")

    def _value(self, metrics: TrainingMetrics) -> float:
        key = {"val_loss": "validation_loss", "val_accuracy": "validation_accuracy"}.get(self.monitor_metric,
                                                                                          self.monitor_metric)
        return float(getattr(metrics, key))

    def save_checkpoint(self, model, metrics: TrainingMetrics, epoch: int, optimizer=None) -> bool:
        v = self._value(metrics)
        better = v > self.best_metric_value if self.maximize_metric else v < self.best_metric_value
        if self.save_best_only and not better:
            return False
        if not self.save_best_only and epoch % self.save_frequency:
            return False
        path = self.generate_checkpoint_filename(epoch, v)
        data = CheckpointData(metadata=ModelMetadata(name=self.model_name), current_epoch=epoch,
                              current_lr=optimizer.get_learning_rate() if optimizer else 0.0,
                              current_metrics=metrics)
        if self.format is SerializationFormat.DLVK_JSON:
            ModelSerializer(SerializationFormat.DLVK_JSON).save_json(model, path, data.metadata)
        else:
            ModelSerializer.save_checkpoint_data(data, path, model, optimizer)
        self.save_metrics(metrics, os.path.join(self.checkpoint_dir, f"{self.model_name}_metrics_{epoch:04d}.json"),
                          epoch)
        self.checkpoint_history.append(path)
        if better:
            self.best_metric_value = v
            self.best_checkpoint_path = path
        self.cleanup_old_checkpoints()
        return True

    def cleanup_old_checkpoints(self) -> None:
        while self.max_checkpoints > 0 and len(self.checkpoint_history) > self.max_checkpoints:
            old = self.checkpoint_history.pop(0)
            if old == self.best_checkpoint_path:
                self.checkpoint_history.append(old)
                if len(self.checkpoint_history) <= self.max_checkpoints:
                    break
                old = self.checkpoint_history.pop(0)
            for p in (old, old.replace("_epoch_", "_metrics_").rsplit(".", 1)[0] + ".json"):
                if os.path.exists(p):
                    os.remove(p)

    def load_checkpoint(self, checkpoint_path: str, model=None, optimizer=None, device=None):
        """Load into `model` (or rebuild one); returns (model, CheckpointData)."""
        if checkpoint_path.endswith(".json"):
            m = ModelSerializer(SerializationFormat.DLVK_JSON).load_json(checkpoint_path, device)
            return m, CheckpointData()
        if model is None:
            model = ModelSerializer().load_binary(checkpoint_path, device)
        data = ModelSerializer.load_checkpoint_data(checkpoint_path, model, optimizer)
        return model, data

    def save_metrics(self, metrics: TrainingMetrics, filepath: str, epoch: int) -> bool:
        with open(filepath, "w") as f:
            json.dump({"epoch": epoch, **metrics.as_dict(), "timestamp": time.time()}, f, indent=1)
        return True

    def get_best_checkpoint_path(self) -> str:
        return self.best_checkpoint_path

    def get_checkpoint_history(self) -> List[str]:
        return list(self.checkpoint_history)

    def list_checkpoints(self) -> List[str]:
        return sorted(glob.glob(os.path.join(self.checkpoint_dir, f"{self.model_name}_epoch_*")))

    def set_checkpoint_directory(self, d: str) -> None:
        self.checkpoint_dir = d
        os.makedirs(d, exist_ok=True)


class ModelVersioning:
    def __init__(self, experiment_dir: str):
        self.experiment_dir = experiment_dir
        self.current_experiment = "default"
        self.experiment_metadata: Dict[str, str] = {}
        os.makedirs(experiment_dir, exist_ok=True)

    def create_experiment(self, name: str, metadata: Optional[Dict[str, str]] = None) -> None:
        self.current_experiment = name
        self.experiment_metadata = dict(metadata or {})
        os.makedirs(self.get_experiment_path(), exist_ok=True)
        with open(os.path.join(self.get_experiment_path(), "experiment.json"), "w") as f:
            json.dump({"name": name, "metadata": self.experiment_metadata, "created": time.time()}, f, indent=1)

    def get_experiment_path(self) -> str:
        return os.path.join(self.experiment_dir, self.current_experiment)

    def _next_tag(self) -> str:
        n = len(self.list_versions()) + 1
        return f"v{n:03d}"

    def save_model_version(self, model, version_tag: Optional[str] = None,
                           metadata: Optional[ModelMetadata] = None, metrics: Optional[dict] = None) -> str:
        tag = version_tag or self._next_tag()
        d = os.path.join(self.get_experiment_path(), tag)
        os.makedirs(d, exist_ok=True)
        path = os.path.join(d, "model.dlvk")
        ModelSerializer().save_binary(model, path, metadata)
        self.save_version_info(tag, (metadata or ModelMetadata()).description, path, metrics)
        return path

    def create_version(self, model, name: str, description: str) -> str:
        return self.save_model_version(model, name, ModelMetadata(name=name, description=description))

    def save_version_info(self, name: str, description: str, model_path: str,
                          metrics: Optional[dict] = None) -> bool:
        with open(os.path.join(os.path.dirname(model_path), "version_info.json"), "w") as f:
            json.dump({"version": name, "description": description, "model_path": model_path,
                       "metrics": metrics or {}, "created": time.time()}, f, indent=1)
        return True

    def load_model_version(self, version_tag: str, device=None):
        return ModelSerializer().load_binary(os.path.join(self.get_experiment_path(), version_tag, "model.dlvk"),
                                             device)

    def list_versions(self) -> List[str]:
        p = self.get_experiment_path()
        if not os.path.isdir(p):
            return []
        return sorted(d for d in os.listdir(p) if os.path.exists(os.path.join(p, d, "version_info.json")))

    def compare_versions(self, a: str, b: str, metric: str = "val_loss") -> dict:
        def info(tag):
            with open(os.path.join(self.get_experiment_path(), tag, "version_info.json")) as f:
                return json.load(f).get("metrics", {})

        ma, mb = info(a), info(b)
        res = {"version_a": a, "version_b": b, "metrics_a": ma, "metrics_b": mb, "better_version": "",
               "comparison_reason": ""}
        if metric in ma and metric in mb:
            lower_better = "loss" in metric
            better = a if ((ma[metric] < mb[metric]) == lower_better) else b
            res["better_version"] = better
            res["comparison_reason"] = f"{metric}: {ma[metric]} vs {mb[metric]}"
        else:
            res["comparison_reason"] = f"metric {metric} missing"
        return res


class ModelCheckpointCallback(TrainingCallback):
    def __init__(self, model, checkpoint_dir: str, model_name: str = "model", optimizer=None,
                 save_best_only: bool = True, monitor_metric: str = "val_loss"):
        self.model = model
        self.optimizer = optimizer
        self.manager = ModelCheckpoint(checkpoint_dir, model_name, save_best_only=save_best_only,
                                       monitor_metric=monitor_metric, maximize_metric="acc" in monitor_metric)

    def on_epoch_end(self, epoch, metrics):
        self.manager.save_checkpoint(self.model, metrics, epoch + 1, self.optimizer)

    def get_checkpoint_manager(self) -> ModelCheckpoint:
        return self.manager


# Factory functions of include/dlvk/training/model_persistence.h:362-381
# (namespace persistence_factory).
def create_checkpoint_callback(model, checkpoint_dir: str = "./checkpoints", model_name: str = "model",
                               optimizer=None) -> ModelCheckpointCallback:
    return ModelCheckpointCallback(model, checkpoint_dir, model_name, optimizer)


def create_versioning_system(experiment_dir: str = "./experiments") -> ModelVersioning:
    return ModelVersioning(experiment_dir)
