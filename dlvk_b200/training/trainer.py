"""`training::Trainer` and `create_trainer` (include/dlvk/training/
trainer.h:19-138, src/training/trainer.cpp).

DataLoader-driven fit / evaluate with callbacks.  The reference reported
random loss and accuracy (trainer.cpp:68,89); here every step is a
captured `TrainStep` that accumulates the loss and the correct-prediction
count on the device, read back once per epoch.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional

import torch

from .. import losses as Lo
from .. import optim as Op
from .callbacks import EarlyStopping, ProgressCallback, TrainingCallback, TrainingMetrics
from .step import TrainStep


def _targets(y: torch.Tensor) -> torch.Tensor:
    return y


class Trainer:
    def __init__(self, model, optimizer, loss_fn, graph: bool = True, scaler=None, regularizer=None):
        self.model = model.build() if hasattr(model, "build") else model
        self.optimizer = optimizer
        self.loss_fn = loss_fn
        self.callbacks: List[TrainingCallback] = []
        self.current_metrics = TrainingMetrics()
        self.history: List[TrainingMetrics] = []
        self.should_stop = False
        self.stop_training = False
        self.graph = graph
        self.scaler = scaler
        self.regularizer = regularizer
        self._steps: Dict[tuple, TrainStep] = {}

    # reference names
    def add_callback(self, cb: TrainingCallback) -> None:
        cb.trainer = self
        self.callbacks.append(cb)

    def get_metrics(self) -> TrainingMetrics:
        return self.current_metrics

    def compute_accuracy(self, predictions: torch.Tensor, targets: torch.Tensor) -> float:
        p = predictions.reshape(-1, predictions.shape[-1]).float().argmax(-1)
        t = targets.reshape(-1, targets.shape[-1]).argmax(-1) if targets.is_floating_point() and \
            targets.dim() > 1 else targets.reshape(-1).long()
        return float((p.cpu() == t.cpu()).float().mean())

    def _step(self, x, y) -> TrainStep:
        key = (tuple(x.shape), x.dtype, tuple(y.shape), y.dtype)
        st = self._steps.get(key)
        if st is None:
            st = TrainStep(self.model, self.loss_fn, self.optimizer, graph=self.graph, metrics=True,
                           scaler=self.scaler, regularizer=self.regularizer)
            self._steps[key] = st
        return st

    def reset_graphs(self) -> None:
        """Drop captured steps (after changing something a graph baked in,
        e.g. a dropout rate)."""
        for st in self._steps.values():
            st.close()
        self._steps.clear()

    def process_batch(self, inputs, targets, training: bool = True) -> TrainingMetrics:
        if training:
            loss = self._step(inputs, targets)(inputs, targets)
            return TrainingMetrics(loss=float(loss))
        m = self._eval_batches([(inputs, targets)])
        return m

    def _collect(self):
        loss = acc_rows = 0.0
        n = rows = 0
        for st in self._steps.values():
            r = st.rows
            l_, a_, n_ = st.epoch_metrics()
            loss += l_ * n_
            acc_rows += a_ * r
            n += n_
            rows += r
        return loss / max(n, 1), acc_rows / max(rows, 1), n

    def fit(self, train_loader, val_loader=None, epochs: int = 1, verbose: bool = True) -> List[TrainingMetrics]:
        if verbose and not any(isinstance(c, ProgressCallback) for c in self.callbacks):
            self.add_callback(ProgressCallback(epochs))
        for c in self.callbacks:
            if hasattr(c, "set_total_epochs"):
                c.set_total_epochs(epochs)
            c.on_train_begin()
        self.should_stop = self.stop_training = False
        for epoch in range(epochs):
            self.model.set_training(True)
            for c in self.callbacks:
                c.on_epoch_begin(epoch)
            t0 = time.perf_counter()
            for bi, (x, y) in enumerate(train_loader):
                for c in self.callbacks:
                    c.on_batch_begin(bi)
                self._step(x, y)(x, y)
            loss, acc, n = self._collect()
            m = TrainingMetrics(loss=loss, accuracy=acc, epoch=epoch,
                                learning_rate=self.optimizer.get_learning_rate())
            if val_loader is not None:
                vm = self.evaluate(val_loader, verbose=False)
                m.validation_loss, m.validation_accuracy = vm.loss, vm.accuracy
            dt = time.perf_counter() - t0
            m.epoch_time_ms, m.samples_per_s = dt * 1e3, (n / dt if dt > 0 else 0.0)
            self.current_metrics = m
            self.history.append(m)
            for c in self.callbacks:
                c.on_epoch_end(epoch, m)
            if hasattr(train_loader, "new_epoch"):
                train_loader.new_epoch()
            if self.stop_training or any(isinstance(c, EarlyStopping) and c.should_stop() for c in self.callbacks):
                self.should_stop = True
                break
        for c in self.callbacks:
            c.on_train_end()
        return self.history

    def _eval_batches(self, batches) -> TrainingMetrics:
        self.model.set_training(False)
        fused = getattr(self.loss_fn, "fuses_softmax", False) and self.model.has_trailing_softmax()
        tot, correct, n, rows = 0.0, 0, 0, 0
        with torch.no_grad():
            for x, y in batches:
                out = self.model.forward_logits(x) if fused else self.model.forward(x)
                yd = y.to(out.device)
                loss, _ = self.loss_fn.value_and_grad(out, yd, from_logits=fused)
                b = x.shape[0]
                tot += float(loss) * b
                n += b
                if out.shape[-1] > 1:
                    p = out.reshape(-1, out.shape[-1]).float().argmax(-1)
                    t = yd.reshape(-1, yd.shape[-1]).argmax(-1) if yd.is_floating_point() else yd.reshape(-1).long()
                    correct += int((p == t).sum())
                    rows += p.numel()
        return TrainingMetrics(loss=tot / max(n, 1), accuracy=correct / max(rows, 1))

    def evaluate(self, data_loader, verbose: bool = True) -> TrainingMetrics:
        m = self._eval_batches(data_loader)
        if verbose:
            print(f"evaluate - loss: {m.loss:.4f} - accuracy: {m.accuracy:.4f}")
        return m

    def close(self):
        self.reset_graphs()


def make_optimizer(name: str, learning_rate: float):
    name = name.lower()
    if name == "sgd":
        return Op.SGD(learning_rate)
    if name == "adam":
        return Op.Adam(learning_rate)
    if name == "rmsprop":
        return Op.RMSprop(learning_rate)
    raise ValueError(f"unknown optimizer '{name}' (sgd, adam, rmsprop)")


def make_loss(name: str):
    name = name.lower()
    if name in ("crossentropy", "cross_entropy", "ce"):
        return Lo.CrossEntropyLoss()
    if name == "mse":
        return Lo.MeanSquaredError()
    if name in ("bce", "binary_crossentropy"):
        return Lo.BinaryCrossEntropyLoss()
    raise ValueError(f"unknown loss '{name}' (mse, crossentropy, bce)")


def create_trainer(model, optimizer_name: str = "adam", learning_rate: float = 0.001,
                   loss_name: str = "crossentropy", **kw) -> Trainer:
    """trainer.cpp:232-265."""
    return Trainer(model, make_optimizer(optimizer_name, learning_rate), make_loss(loss_name), **kw)
