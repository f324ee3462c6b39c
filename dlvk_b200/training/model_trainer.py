"""`ModelTrainer` (include/dlvk/model/model.h:115-143, src/model/model.cpp:
211-536): compile / fit / evaluate / predict.

Fixes relative to the reference: batches are slices of the data (the
reference copied the whole dataset into every batch, model.cpp:499-536),
`validation_split` really holds out the last fraction (model.cpp:441-497
did not split), the optimizer set in compile() is the one that updates the
weights (Sequential::update_parameters always applied plain SGD), and
full-size batches run as one captured CUDA graph per step.
"""
from __future__ import annotations

import time
from typing import List, Optional

import torch

from .callbacks import TrainingCallback, TrainingMetrics
from .step import TrainStep


def _targets_to_labels(y: torch.Tensor) -> torch.Tensor:
    if y.is_floating_point() and y.dim() >= 2 and y.shape[-1] > 1:
        return y.argmax(-1)
    return y.reshape(-1).long() if not y.is_floating_point() else y.reshape(-1).round().long()


class ModelTrainer:
    def __init__(self, model):
        self.model = model
        self.optimizer = None
        self.loss_function = None
        self.callbacks: List[TrainingCallback] = []
        self.stop_training = False
        self.history: List[TrainingMetrics] = []
        self._steps = {}
        self.use_graph = True
        self.scaler = None        # optional GradientScaler
        self.regularizer = None   # optional RegularizationManager

    # -- reference API -----------------------------------------------------------
    def compile(self, optimizer, loss_function):
        self.optimizer = optimizer
        self.loss_function = loss_function
        self._steps = {}

    def add_callback(self, cb: TrainingCallback):
        cb.trainer = self
        self.callbacks.append(cb)

    def get_optimizer(self):
        return self.optimizer

    def _step_for(self, x, y) -> TrainStep:
        key = (tuple(x.shape), x.dtype, tuple(y.shape), y.dtype)
        st = self._steps.get(key)
        if st is None:
            st = TrainStep(self.model, self.loss_function, self.optimizer, graph=self.use_graph, metrics=True,
                           scaler=self.scaler, regularizer=self.regularizer)
            self._steps[key] = st
        return st

    def collect_metrics(self):
        """(mean loss, accuracy, samples) over every step since the last call."""
        loss = acc_rows = 0.0
        n = rows = 0
        for st in self._steps.values():
            r = st.rows
            m_loss, m_acc, m_n = st.epoch_metrics()
            loss += m_loss * m_n
            acc_rows += m_acc * r
            n += m_n
            rows += r
        return loss / max(n, 1), acc_rows / max(rows, 1), n

    @staticmethod
    def split_data(x, y, validation_split: float):
        if validation_split <= 0:
            return x, y, None, None
        n = x.shape[0]
        nv = int(round(n * validation_split))
        nt = n - nv
        return x[:nt], y[:nt], x[nt:], y[nt:]

    @staticmethod
    def create_batches(x, y, batch_size: int):
        n = x.shape[0]
        return [(x[i:i + batch_size], y[i:i + batch_size]) for i in range(0, n, batch_size)]

    def calculate_accuracy(self, predictions: torch.Tensor, targets: torch.Tensor) -> float:
        pred = predictions.reshape(-1, predictions.shape[-1]).float().argmax(-1).cpu()
        lab = _targets_to_labels(targets.cpu() if targets.is_floating_point() else targets.cpu())
        return float((pred == lab.reshape(-1)).float().mean()) if lab.numel() == pred.numel() else 0.0

    def fit(self, x_train, y_train, epochs: int, batch_size: int = 32, validation_split: float = 0.0,
            verbose: bool = True, shuffle: bool = True, seed: int = 0, log_every: int = 0) -> List[TrainingMetrics]:
        from .callbacks import ProgressCallback

        if self.optimizer is None or self.loss_function is None:
            raise RuntimeError("compile() the trainer first")
        x_tr, y_tr, x_val, y_val = self.split_data(x_train, y_train, validation_split)
        if verbose and not any(isinstance(c, ProgressCallback) for c in self.callbacks):
            self.add_callback(ProgressCallback(epochs))
        for c in self.callbacks:
            if hasattr(c, "set_total_epochs"):
                c.set_total_epochs(epochs)
            c.on_train_begin()
        self.stop_training = False
        self.model.set_training(True)
        g = torch.Generator().manual_seed(seed)
        pin = self.model.dev.is_cuda
        for epoch in range(epochs):
            for c in self.callbacks:
                c.on_epoch_begin(epoch)
            t0 = time.perf_counter()
            n = x_tr.shape[0]
            order = torch.randperm(n, generator=g) if shuffle else torch.arange(n)
            for bi, s in enumerate(range(0, n, batch_size)):
                idx = order[s:s + batch_size]
                xb, yb = x_tr[idx], y_tr[idx]
                if pin:
                    xb, yb = xb.pin_memory(), yb.pin_memory()
                for c in self.callbacks:
                    c.on_batch_begin(bi)
                step = self._step_for(xb, yb)
                loss = step(xb, yb)
                if log_every and (bi + 1) % log_every == 0:
                    m = TrainingMetrics(loss=float(loss), epoch=epoch, batch=bi,
                                        learning_rate=self.optimizer.get_learning_rate())
                    for c in self.callbacks:
                        c.on_batch_end(bi, m)
            ep_loss, train_acc, seen = self.collect_metrics()
            metrics = TrainingMetrics(loss=ep_loss, accuracy=train_acc, epoch=epoch,
                                      learning_rate=self.optimizer.get_learning_rate())
            if x_val is not None and x_val.shape[0] > 0:
                vm = self.evaluate(x_val, y_val, batch_size)
                metrics.validation_loss, metrics.validation_accuracy = vm.loss, vm.accuracy
                self.model.set_training(True)
            dt = time.perf_counter() - t0
            metrics.epoch_time_ms = dt * 1e3
            metrics.samples_per_s = seen / dt if dt > 0 else 0.0
            self.history.append(metrics)
            for c in self.callbacks:
                c.on_epoch_end(epoch, metrics)
            if self.stop_training:
                break
        for c in self.callbacks:
            c.on_train_end()
        return self.history

    def evaluate(self, x_test, y_test, batch_size: int = 32) -> TrainingMetrics:
        self.model.set_training(False)
        tot_loss, total, correct = 0.0, 0, 0
        fused = getattr(self.loss_function, "fuses_softmax", False) and self.model.has_trailing_softmax()
        with torch.no_grad():
            for xb, yb in self.create_batches(x_test, y_test, batch_size):
                out = self.model.forward_logits(xb) if fused else self.model.forward(xb)
                yb_d = yb.to(out.device)
                loss, _ = self.loss_function.value_and_grad(out, yb_d, from_logits=fused)
                tot_loss += float(loss) * xb.shape[0]
                if out.shape[-1] > 1:
                    pred = out.reshape(-1, out.shape[-1]).float().argmax(-1).cpu()
                    lab = _targets_to_labels(yb.cpu())
                    correct += int((pred == lab.reshape(-1)).sum())
                total += xb.shape[0]
        n = max(total, 1)
        return TrainingMetrics(loss=tot_loss / n, accuracy=correct / n)

    def predict(self, x, batch_size: int = 32) -> torch.Tensor:
        self.model.set_training(False)
        outs = []
        with torch.no_grad():
            for s in range(0, x.shape[0], batch_size):
                outs.append(self.model.forward(x[s:s + batch_size]))
        return torch.cat(outs) if outs else torch.empty(0)
