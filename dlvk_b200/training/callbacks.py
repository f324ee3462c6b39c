"""Training metrics and callbacks (include/dlvk/model/model.h:93-113,
include/dlvk/model/callbacks.h:10-117, src/model/callbacks.cpp).

Metric values are real (the reference's training::Trainer reported rand(),
src/training/trainer.cpp:68,89).  Losses stay on the device during an epoch
and are read back once per epoch (or every `log_every` batches), so
callbacks do not force a host synchronisation per step.
"""
from __future__ import annotations

import csv
import math
import os
import sys
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class TrainingMetrics:
    loss: float = 0.0
    accuracy: float = 0.0
    validation_loss: float = 0.0
    validation_accuracy: float = 0.0
    epoch: int = 0
    batch: int = 0
    learning_rate: float = 0.0
    epoch_time_ms: float = 0.0
    samples_per_s: float = 0.0

    # training::TrainingMetrics spellings (include/dlvk/training/trainer.h:19-35)
    @property
    def train_loss(self):
        return self.loss

    @property
    def train_accuracy(self):
        return self.accuracy

    @property
    def val_loss(self):
        return self.validation_loss

    @property
    def val_accuracy(self):
        return self.validation_accuracy

    def as_dict(self) -> Dict[str, float]:
        return {"epoch": self.epoch, "loss": self.loss, "accuracy": self.accuracy,
                "val_loss": self.validation_loss, "val_accuracy": self.validation_accuracy,
                "learning_rate": self.learning_rate, "epoch_time_ms": self.epoch_time_ms,
                "samples_per_s": self.samples_per_s}


class TrainingCallback:
    trainer = None  # set by the trainer

    def on_train_begin(self):
        pass

    def on_train_end(self):
        pass

    def on_epoch_begin(self, epoch: int):
        pass

    def on_epoch_end(self, epoch: int, metrics: TrainingMetrics):
        pass

    def on_batch_begin(self, batch: int):
        pass

    def on_batch_end(self, batch: int, metrics: TrainingMetrics):
        pass

    # training::TrainingCallback spellings
    def on_training_begin(self):
        self.on_train_begin()

    def on_training_end(self):
        self.on_train_end()


def _monitored(metrics: TrainingMetrics, monitor: str) -> float:
    key = {"loss": "loss", "accuracy": "accuracy", "val_loss": "validation_loss",
           "val_accuracy": "validation_accuracy", "validation_loss": "validation_loss",
           "validation_accuracy": "validation_accuracy"}.get(monitor, monitor)
    return float(getattr(metrics, key))


def _mode_for(monitor: str, mode: str) -> str:
    if mode != "auto":
        return mode
    return "max" if "acc" in monitor else "min"


class ProgressCallback(TrainingCallback):
    """Per-epoch progress with epoch time (src/model/callbacks.cpp:18-41)."""

    def __init__(self, total_epochs: int = 0, print_every: int = 1, stream=None):
        self.total_epochs = total_epochs
        self.print_every = max(1, print_every)
        self.stream = stream or sys.stdout
        self._t0 = 0.0
        self.lines: List[str] = []

    def set_total_epochs(self, epochs: int):
        self.total_epochs = epochs

    def set_batches_per_epoch(self, batches: int):
        self.batches = batches

    def on_epoch_begin(self, epoch):
        self._t0 = time.perf_counter()

    def on_epoch_end(self, epoch, metrics):
        if (epoch + 1) % self.print_every:
            return
        ms = (time.perf_counter() - self._t0) * 1e3
        line = (f"Epoch {epoch + 1}/{self.total_epochs or '?'} - {ms:.1f}ms - loss: {metrics.loss:.4f} - "
                f"accuracy: {metrics.accuracy:.4f}")
        if metrics.validation_loss:
            line += f" - val_loss: {metrics.validation_loss:.4f} - val_accuracy: {metrics.validation_accuracy:.4f}"
        self.lines.append(line)
        print(line, file=self.stream, flush=True)


class ModelCheckpoint(TrainingCallback):
    """Save weights when the monitored value improves (or every epoch)
    (src/model/callbacks.cpp:77-102).  `{epoch}` in the path is formatted."""

    def __init__(self, filepath: str, monitor: str = "val_loss", save_best_only: bool = True, mode: str = "auto",
                 verbose: bool = False, save_optimizer: bool = True):
        self.filepath, self.monitor, self.save_best_only = filepath, monitor, save_best_only
        self.mode = _mode_for(monitor, mode)
        self.best = math.inf if self.mode == "min" else -math.inf
        self.verbose = verbose
        self.save_optimizer = save_optimizer
        self.saved: List[str] = []

    def is_improvement(self, v: float) -> bool:
        return v < self.best if self.mode == "min" else v > self.best

    def get_monitored_value(self, metrics):
        return _monitored(metrics, self.monitor)

    def on_epoch_end(self, epoch, metrics):
        v = self.get_monitored_value(metrics)
        if self.save_best_only and not self.is_improvement(v):
            return
        self.best = v if self.is_improvement(v) else self.best
        path = self.filepath.format(epoch=epoch + 1)
        tr = self.trainer
        opt = tr.optimizer if (tr is not None and self.save_optimizer) else None
        tr.model.save_weights(path, optimizer=opt, extra_meta={"epoch": epoch + 1, **metrics.as_dict()})
        self.saved.append(path)
        if self.verbose:
            print(f"Epoch {epoch + 1}: {self.monitor} = {v:.5f}, saved {path}")


class EarlyStopping(TrainingCallback):
    """Stop after `patience` epochs without improvement by `min_delta`
    (src/model/callbacks.cpp:122-171)."""

    def __init__(self, monitor: str = "val_loss", patience: int = 5, min_delta: float = 0.0, mode: str = "auto",
                 restore_best_weights: bool = False):
        self.monitor, self.patience, self.min_delta = monitor, patience, min_delta
        self.mode = _mode_for(monitor, mode)
        self.restore_best_weights = restore_best_weights
        self.wait = 0
        self.best = math.inf if self.mode == "min" else -math.inf
        self.stopped_epoch = -1
        self._best_state = None

    def on_train_begin(self):
        self.wait = 0
        self.best = math.inf if self.mode == "min" else -math.inf
        self.stopped_epoch = -1

    def is_improvement(self, v: float) -> bool:
        return v < self.best - self.min_delta if self.mode == "min" else v > self.best + self.min_delta

    def get_monitored_value(self, metrics):
        return _monitored(metrics, self.monitor)

    def should_stop(self) -> bool:
        return self.stopped_epoch >= 0

    def on_epoch_end(self, epoch, metrics):
        v = self.get_monitored_value(metrics)
        if self.is_improvement(v):
            self.best = v
            self.wait = 0
            if self.restore_best_weights and self.trainer is not None:
                self._best_state = self.trainer.model.store.master.detach().clone()
        else:
            self.wait += 1
            if self.wait >= self.patience:
                self.stopped_epoch = epoch
                if self.trainer is not None:
                    self.trainer.stop_training = True

    def on_train_end(self):
        if self._best_state is not None and self.trainer is not None and self.should_stop():
            self.trainer.model.store.master.copy_(self._best_state)
            self.trainer.model.store.sync_value()


EarlyStoppingCallback = EarlyStopping


class ReduceLROnPlateau(TrainingCallback):
    """lr *= factor after `patience` epochs without improvement, floored at
    min_lr (src/model/callbacks.cpp:174-233)."""

    def __init__(self, monitor: str = "val_loss", factor: float = 0.1, patience: int = 10, min_lr: float = 0.0,
                 mode: str = "auto", min_delta: float = 1e-4, verbose: bool = False):
        self.monitor, self.factor, self.patience, self.min_lr = monitor, factor, patience, min_lr
        self.mode = _mode_for(monitor, mode)
        self.min_delta = min_delta
        self.verbose = verbose
        self.wait = 0
        self.best = math.inf if self.mode == "min" else -math.inf

    def on_train_begin(self):
        self.wait = 0
        self.best = math.inf if self.mode == "min" else -math.inf

    def is_improvement(self, v):
        return v < self.best - self.min_delta if self.mode == "min" else v > self.best + self.min_delta

    def get_monitored_value(self, metrics):
        return _monitored(metrics, self.monitor)

    def on_epoch_end(self, epoch, metrics):
        v = self.get_monitored_value(metrics)
        if self.is_improvement(v):
            self.best = v
            self.wait = 0
            return
        self.wait += 1
        if self.wait >= self.patience and self.trainer is not None:
            opt = self.trainer.optimizer
            new = max(self.min_lr, opt.get_learning_rate() * self.factor)
            if new < opt.get_learning_rate():
                opt.set_learning_rate(new)
                if self.verbose:
                    print(f"Epoch {epoch + 1}: reducing learning rate to {new:.3g}")
            self.wait = 0


class CSVLogger(TrainingCallback):
    """epoch,loss,accuracy,val_loss,val_accuracy rows (src/model/callbacks.cpp:236-265)."""

    FIELDS = ["epoch", "loss", "accuracy", "val_loss", "val_accuracy"]

    def __init__(self, filename: str, append: bool = False):
        self.filename, self.append = filename, append

    def on_train_begin(self):
        if not self.append or not os.path.exists(self.filename):
            with open(self.filename, "w", newline="") as f:
                csv.writer(f).writerow(self.FIELDS)

    def on_epoch_end(self, epoch, metrics):
        with open(self.filename, "a", newline="") as f:
            csv.writer(f).writerow([epoch + 1, f"{metrics.loss:.6f}", f"{metrics.accuracy:.6f}",
                                    f"{metrics.validation_loss:.6f}", f"{metrics.validation_accuracy:.6f}"])


class LambdaCallback(TrainingCallback):
    def __init__(self, on_epoch_end=None, on_batch_end=None):
        self._e, self._b = on_epoch_end, on_batch_end

    def on_epoch_end(self, epoch, metrics):
        if self._e:
            self._e(epoch, metrics)

    def on_batch_end(self, batch, metrics):
        if self._b:
            self._b(batch, metrics)
