"""Advanced training (include/dlvk/training/advanced_training.h:21-330,
src/training/advanced_training.cpp).

`AdvancedTrainer` composes what the reference's config names -- mixed
precision (device loss scaler), regularisation (fused L1/L2 kernel),
learning-rate schedules, gradient clipping, early stopping, best-model
checkpointing, validation frequency, logging and training curves -- on top
of the captured `TrainStep`.  The reference left fit / process_epoch /
process_batch / evaluate empty (advanced_training.cpp:96-140).

Schedulers follow advanced_training.cpp:13-67: cosine annealing with
`min_lr` as a fraction of the initial rate; one-cycle linear up for
`pct_start`% of the steps from max*initial_ratio then linear down to
max*final_ratio; reduce-on-plateau with relative threshold, patience and
cooldown (the reference tracked `best` with max() in both modes, so in
"min" mode it never improved; here improvement is mode-aware).
"""
from __future__ import annotations

import enum
import json
import math
import os
import random
import time
from dataclasses import asdict, dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

from .. import optim as Op
from .callbacks import EarlyStopping, TrainingCallback, TrainingMetrics
from .mixed_precision import MixedPrecisionTrainer, PrecisionMode
from .regularization import create_comprehensive_regularization
from .trainer import Trainer, make_loss, make_optimizer


class LRScheduleType(enum.Enum):
    CONSTANT = 0
    STEP_DECAY = 1
    EXPONENTIAL = 2
    COSINE_ANNEALING = 3
    REDUCE_ON_PLATEAU = 4
    CYCLIC = 5
    ONE_CYCLE = 6


class LearningRateScheduler:
    def get_lr(self, step: int, current_lr: float, validation_metric: float = 0.0) -> float:
        raise NotImplementedError

    def step(self, validation_metric: float = 0.0) -> None:
        pass

    def reset(self) -> None:
        pass


class ConstantScheduler(LearningRateScheduler):
    def get_lr(self, step, current_lr, validation_metric=0.0):
        return current_lr


class StepDecayScheduler(LearningRateScheduler):
    def __init__(self, initial_lr: float, factor: float = 0.1, step_size: int = 30):
        self.initial_lr, self.factor, self.step_size = initial_lr, factor, step_size
        self.current_step = 0

    def get_lr(self, step, current_lr, validation_metric=0.0):
        return self.initial_lr * self.factor ** (self.current_step // self.step_size)

    def step(self, validation_metric=0.0):
        self.current_step += 1

    def reset(self):
        self.current_step = 0


class ExponentialScheduler(StepDecayScheduler):
    def get_lr(self, step, current_lr, validation_metric=0.0):
        return self.initial_lr * self.factor ** self.current_step


class CosineAnnealingScheduler(LearningRateScheduler):
    def __init__(self, initial_lr: float, min_lr: float, max_steps: int):
        self.initial_lr, self.min_lr, self.max_steps = float(initial_lr), float(min_lr), int(max_steps)
        self.current_step = 0

    def get_lr(self, step, current_lr, validation_metric=0.0):
        t = min(self.current_step, self.max_steps)
        decay = 0.5 * (1.0 + math.cos(math.pi * t / self.max_steps))
        return self.initial_lr * ((1.0 - self.min_lr) * decay + self.min_lr)

    def step(self, validation_metric=0.0):
        self.current_step += 1

    def reset(self):
        self.current_step = 0


class CyclicScheduler(LearningRateScheduler):
    """Triangular cycle between base and max over 2*half_cycle steps."""

    def __init__(self, base_lr: float, max_lr: float, half_cycle: int = 100):
        self.base_lr, self.max_lr, self.half = base_lr, max_lr, max(1, half_cycle)
        self.current_step = 0

    def get_lr(self, step, current_lr, validation_metric=0.0):
        pos = self.current_step % (2 * self.half)
        frac = pos / self.half if pos < self.half else 2.0 - pos / self.half
        return self.base_lr + (self.max_lr - self.base_lr) * frac

    def step(self, validation_metric=0.0):
        self.current_step += 1

    def reset(self):
        self.current_step = 0


class OneCycleScheduler(LearningRateScheduler):
    def __init__(self, max_lr: float, total_steps: int, initial_lr_ratio: float = 0.1,
                 final_lr_ratio: float = 0.01, pct_start: int = 30):
        self.max_lr, self.total_steps, self.pct_start = float(max_lr), int(total_steps), int(pct_start)
        self.initial_lr = self.max_lr * initial_lr_ratio
        self.final_lr = self.max_lr * final_lr_ratio
        self.current_step = 0

    def get_lr(self, step, current_lr, validation_metric=0.0):
        up = max(1, int(self.total_steps * (self.pct_start / 100.0)))
        down = max(1, self.total_steps - up)
        t = self.current_step
        if t <= up:
            return self.initial_lr + (self.max_lr - self.initial_lr) * t / up
        return max(self.final_lr, self.max_lr - (self.max_lr - self.final_lr) * (t - up) / down)

    def step(self, validation_metric=0.0):
        self.current_step += 1

    def reset(self):
        self.current_step = 0


class ReduceOnPlateauScheduler(LearningRateScheduler):
    def __init__(self, factor: float = 0.1, patience: int = 10, threshold: float = 1e-4, cooldown: int = 0,
                 min_lr: float = 0.0, mode_max: bool = False):
        self.factor, self.patience, self.threshold = factor, patience, threshold
        self.cooldown, self.min_lr, self.mode_max = cooldown, min_lr, mode_max
        self.reset()

    def _improved(self, v: float) -> bool:
        if math.isinf(self.best):
            return True
        if self.mode_max:
            return v > self.best * (1.0 + self.threshold) if self.best >= 0 else v > self.best * (1 - self.threshold)
        return v < self.best * (1.0 - self.threshold) if self.best >= 0 else v < self.best * (1 + self.threshold)

    def get_lr(self, step, current_lr, validation_metric=0.0):
        if self.cooldown_count > 0:
            self.cooldown_count -= 1
            return current_lr
        if self._improved(validation_metric):
            self.best = validation_metric
            self.wait = 0
        else:
            self.wait += 1
        if self.wait >= self.patience:
            self.wait = 0
            self.cooldown_count = self.cooldown
            return max(current_lr * self.factor, self.min_lr)
        return current_lr

    def step(self, validation_metric=0.0):
        pass

    def reset(self):
        self.best = -math.inf if self.mode_max else math.inf
        self.wait = 0
        self.cooldown_count = 0


@dataclass
class AdvancedTrainingConfig:
    use_mixed_precision: bool = False
    precision_mode: PrecisionMode = PrecisionMode.MIXED
    enable_gradient_scaling: bool = True

    use_regularization: bool = False
    l2_lambda: float = 0.01
    weight_decay: float = 0.0001
    use_dropout_scheduling: bool = False

    lr_schedule: LRScheduleType = LRScheduleType.CONSTANT
    lr_decay_factor: float = 0.1
    lr_decay_patience: int = 10
    lr_min: float = 1e-7

    use_gradient_clipping: bool = False
    gradient_clip_value: float = 1.0
    gradient_clip_by_norm: bool = True

    use_early_stopping: bool = True
    early_stopping_patience: int = 15
    save_best_model: bool = True
    checkpoint_dir: str = "./checkpoints"

    validation_split: float = 0.2
    validation_frequency: int = 1

    verbose_training: bool = True
    log_frequency: int = 10
    save_training_curves: bool = True


@dataclass
class TrainingStatistics:
    total_training_time: float = 0.0
    average_epoch_time: float = 0.0
    best_validation_loss: float = 0.0
    best_validation_accuracy: float = 0.0
    best_epoch: int = 0
    total_epochs_trained: int = 0
    converged: bool = False
    memory_savings_ratio: float = 0.0
    training_speedup: float = 0.0
    final_l1_loss: float = 0.0
    final_l2_loss: float = 0.0
    final_weight_decay: float = 0.0


class AdvancedTrainer:
    def __init__(self, model, optimizer, loss_fn, config: Optional[AdvancedTrainingConfig] = None):
        self.model = model.build() if hasattr(model, "build") else model
        self.optimizer = optimizer
        self.loss_fn = loss_fn
        self.config = config or AdvancedTrainingConfig()
        self.callbacks: List[TrainingCallback] = []
        self.history: List[TrainingMetrics] = []
        self.best_validation_loss = math.inf
        self.best_validation_accuracy = 0.0
        self.best_epoch = 0
        self.epochs_without_improvement = 0
        self.should_stop = False
        self._setup()

    # ------------------------------------------------------------------ setup
    def _setup(self):
        c = self.config
        self.mp_trainer = None
        scaler = None
        if c.use_mixed_precision:
            self.mp_trainer = MixedPrecisionTrainer(c.precision_mode, device=self.model.dev.device)
            if c.enable_gradient_scaling:
                scaler = self.mp_trainer.get_context().get_scaler()
        self.regularization = None
        if c.use_regularization:
            self.regularization = create_comprehensive_regularization(c.l2_lambda, c.weight_decay, True,
                                                                      c.l2_lambda * 0.1)
        if c.use_gradient_clipping:
            if c.gradient_clip_by_norm:
                self.optimizer.set_gradient_clipping(max_norm=c.gradient_clip_value)
            elif scaler is None:
                self.optimizer.set_gradient_clipping(clip_value=c.gradient_clip_value)
        lr0 = self.optimizer.get_learning_rate()
        s = c.lr_schedule
        if s is LRScheduleType.COSINE_ANNEALING:
            self.lr_scheduler = CosineAnnealingScheduler(lr0, 1e-6, 100)
        elif s is LRScheduleType.STEP_DECAY:
            self.lr_scheduler = StepDecayScheduler(lr0, c.lr_decay_factor, max(1, c.lr_decay_patience))
        elif s is LRScheduleType.EXPONENTIAL:
            self.lr_scheduler = ExponentialScheduler(lr0, 1.0 - c.lr_decay_factor * 0.1)
        elif s is LRScheduleType.REDUCE_ON_PLATEAU:
            self.lr_scheduler = ReduceOnPlateauScheduler(c.lr_decay_factor, c.lr_decay_patience, min_lr=c.lr_min)
        elif s is LRScheduleType.CYCLIC:
            self.lr_scheduler = CyclicScheduler(lr0 * 0.1, lr0)
        elif s is LRScheduleType.ONE_CYCLE:
            self.lr_scheduler = OneCycleScheduler(lr0, 100)
        else:
            self.lr_scheduler = None
        self.trainer = Trainer(self.model, self.optimizer, self.loss_fn, scaler=scaler,
                               regularizer=self.regularization)
        for cb in self.callbacks:
            self.trainer.add_callback(cb)

    def update_config(self, config: AdvancedTrainingConfig) -> None:
        self.config = config
        self.trainer.close()
        self._setup()

    def get_config(self) -> AdvancedTrainingConfig:
        return self.config

    def add_callback(self, cb: TrainingCallback) -> None:
        self.callbacks.append(cb)
        self.trainer.add_callback(cb)

    def get_training_history(self) -> List[TrainingMetrics]:
        return self.history

    # ------------------------------------------------------------------ loop
    def update_learning_rate(self, validation_metric: float) -> None:
        if self.lr_scheduler is None:
            return
        lr = self.lr_scheduler.get_lr(len(self.history), self.optimizer.get_learning_rate(), validation_metric)
        self.lr_scheduler.step(validation_metric)
        self.optimizer.set_learning_rate(max(lr, self.config.lr_min))

    def save_checkpoint(self, epoch: int, is_best: bool = False) -> str:
        os.makedirs(self.config.checkpoint_dir, exist_ok=True)
        name = "best_model.dlvk" if is_best else f"checkpoint_epoch_{epoch + 1:04d}.dlvk"
        path = os.path.join(self.config.checkpoint_dir, name)
        meta = self.history[-1].as_dict() if self.history else {}
        self.model.save_weights(path, optimizer=self.optimizer, extra_meta={"epoch": epoch + 1, **meta})
        return path

    def log_metrics(self, m: TrainingMetrics, is_validation: bool = False) -> None:
        if self.config.verbose_training:
            tag = "val" if is_validation else "train"
            print(f"[{tag}] epoch {m.epoch + 1}: loss {m.loss:.4f} acc {m.accuracy:.4f} "
                  f"val_loss {m.validation_loss:.4f} val_acc {m.validation_accuracy:.4f} lr {m.learning_rate:.3g}")

    def process_epoch(self, train_loader, val_loader, epoch: int) -> TrainingMetrics:
        tr = self.trainer
        self.model.set_training(True)
        t0 = time.perf_counter()
        for x, y in train_loader:
            tr._step(x, y)(x, y)
        loss, acc, n = tr._collect()
        m = TrainingMetrics(loss=loss, accuracy=acc, epoch=epoch, learning_rate=self.optimizer.get_learning_rate())
        if val_loader is not None and (epoch + 1) % max(1, self.config.validation_frequency) == 0:
            vm = tr.evaluate(val_loader, verbose=False)
            m.validation_loss, m.validation_accuracy = vm.loss, vm.accuracy
        dt = time.perf_counter() - t0
        m.epoch_time_ms, m.samples_per_s = dt * 1e3, n / dt if dt > 0 else 0.0
        if hasattr(train_loader, "new_epoch"):
            train_loader.new_epoch()
        return m

    def fit(self, train_loader, val_loader=None, epochs: int = 1) -> List[TrainingMetrics]:
        for cb in self.callbacks:
            cb.on_train_begin()
        t_start = time.perf_counter()
        self.should_stop = False
        for epoch in range(epochs):
            for cb in self.callbacks:
                cb.on_epoch_begin(epoch)
            m = self.process_epoch(train_loader, val_loader, epoch)
            self.history.append(m)
            monitored = m.validation_loss if val_loader is not None else m.loss
            improved = monitored < self.best_validation_loss
            if improved:
                self.best_validation_loss = monitored
                self.best_validation_accuracy = m.validation_accuracy
                self.best_epoch = epoch
                self.epochs_without_improvement = 0
                if self.config.save_best_model:
                    self.save_checkpoint(epoch, is_best=True)
            else:
                self.epochs_without_improvement += 1
            self.update_learning_rate(monitored)
            self.log_metrics(m)
            for cb in self.callbacks:
                cb.on_epoch_end(epoch, m)
            if (self.config.use_early_stopping and self.epochs_without_improvement >= self.config.early_stopping_patience) \
                    or self.trainer.stop_training:
                self.should_stop = True
                break
        self.total_time = time.perf_counter() - t_start
        for cb in self.callbacks:
            cb.on_train_end()
        if self.config.save_training_curves:
            os.makedirs(self.config.checkpoint_dir, exist_ok=True)
            with open(os.path.join(self.config.checkpoint_dir, "training_curves.json"), "w") as f:
                json.dump([h.as_dict() for h in self.history], f, indent=1)
        return self.history

    def evaluate(self, data_loader) -> TrainingMetrics:
        return self.trainer.evaluate(data_loader, verbose=False)

    def get_statistics(self) -> TrainingStatistics:
        st = TrainingStatistics()
        n = len(self.history)
        st.total_training_time = getattr(self, "total_time", 0.0)
        st.average_epoch_time = sum(h.epoch_time_ms for h in self.history) / max(n, 1) / 1e3
        st.best_validation_loss = self.best_validation_loss if n else 0.0
        st.best_validation_accuracy = self.best_validation_accuracy
        st.best_epoch = self.best_epoch
        st.total_epochs_trained = n
        st.converged = self.should_stop
        if self.mp_trainer is not None:
            st.memory_savings_ratio = self.mp_trainer.get_context().estimate_memory_savings()
        if self.regularization is not None:
            gl1, gl2, ll1, ll2 = self.regularization.combined()
            w = self.model.store.master
            st.final_l1_loss = float(ll1 * w.abs().sum())
            st.final_l2_loss = float(0.5 * ll2 * (w * w).sum())
            st.final_weight_decay = self.config.weight_decay
        return st

    def close(self):
        self.trainer.close()


def create_advanced_trainer(model, optimizer_name: str = "adam", learning_rate: float = 0.001,
                            loss_name: str = "crossentropy",
                            config: Optional[AdvancedTrainingConfig] = None) -> AdvancedTrainer:
    return AdvancedTrainer(model, make_optimizer(optimizer_name, learning_rate), make_loss(loss_name), config)


# ---------------------------------------------------------------- hyper-parameter search
@dataclass
class HyperparameterRange:
    min_value: float
    max_value: float
    log_scale: bool = False


@dataclass
class HyperparameterConfig:
    ranges: Dict[str, HyperparameterRange] = field(default_factory=dict)
    n_trials: int = 100
    max_epochs_per_trial: int = 10
    optimization_metric: str = "val_loss"
    maximize_metric: bool = False


@dataclass
class HyperparameterResult:
    best_params: Dict[str, float] = field(default_factory=dict)
    best_score: float = 0.0
    all_results: List[Tuple[Dict[str, float], float]] = field(default_factory=list)


def random_search(objective_fn: Callable[[Dict[str, float]], float], config: HyperparameterConfig,
                  seed: int = 0) -> HyperparameterResult:
    """Random search over the configured ranges (log-uniform where asked).
    The reference passed an empty parameter map to every trial
    (advanced_training.cpp:148-172)."""
    rng = random.Random(seed)
    res = HyperparameterResult()
    for trial in range(config.n_trials):
        params = {}
        for name, r in config.ranges.items():
            if r.log_scale:
                lo, hi = math.log(r.min_value), math.log(r.max_value)
                params[name] = math.exp(rng.uniform(lo, hi))
            else:
                params[name] = rng.uniform(r.min_value, r.max_value)
        score = float(objective_fn(params))
        better = score > res.best_score if config.maximize_metric else score < res.best_score
        if trial == 0 or better:
            res.best_score, res.best_params = score, dict(params)
        res.all_results.append((params, score))
    return res
