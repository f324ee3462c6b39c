"""Regularisation (include/dlvk/training/regularization.h:15-250,
src/training/regularization.cpp).

Math follows regularization.cpp:28-155: L1 loss lambda*sum|w| with
gradient lambda*sign(w); L2 loss 0.5*lambda*sum w^2 with gradient lambda*w;
ElasticNet = L1(lambda*r) + L2(lambda*(1-r)); WeightDecay adds decay*w to
the gradient (loss 0) or shrinks w by (1 - lr*decay).

On the GPU a `RegularizationManager` collapses every regulariser into one
(l1, l2) pair and applies it with ONE fused kernel per contiguous run of
decayed parameters of the model's flat store (`regularize` in
train_aux.cu), optionally accumulating the penalty into a device scalar —
so it runs inside a captured training-step graph.  The per-tensor
`compute_loss` / `compute_gradients` API of the reference is kept for
tensors a user passes explicitly.
"""
from __future__ import annotations

import enum
from typing import List, Optional, Sequence, Tuple

import torch

from ..ops import core as K


class RegularizationType(enum.Enum):
    NONE = 0
    L1 = 1
    L2 = 2
    ELASTIC_NET = 3
    DROPOUT = 4
    BATCH_NORM = 5
    WEIGHT_DECAY = 6


class Regularizer:
    name = "regularizer"
    kind = RegularizationType.NONE

    def coefficients(self) -> Tuple[float, float]:
        """(l1, l2) with gradient l1*sign(w) + l2*w and loss l1|w| + 0.5 l2 w^2."""
        raise NotImplementedError

    def counts_in_loss(self) -> bool:
        return True

    def compute_loss(self, weights: Sequence[torch.Tensor]) -> float:
        l1, l2 = self.coefficients()
        if not self.counts_in_loss():
            return 0.0
        tot = 0.0
        for w in weights:
            wf = w.detach().float()
            tot += float(l1 * wf.abs().sum() + 0.5 * l2 * (wf * wf).sum())
        return tot

    def compute_gradients(self, weights: Sequence[torch.Tensor]) -> List[torch.Tensor]:
        l1, l2 = self.coefficients()
        return [l1 * torch.sign(w.detach().float()) + l2 * w.detach().float() for w in weights]

    def get_strength(self) -> float:
        return self.strength

    def set_strength(self, strength: float) -> None:
        self.strength = float(strength)


class L1Regularizer(Regularizer):
    name, kind = "L1", RegularizationType.L1

    def __init__(self, lambda_: float = 0.01):
        self.strength = float(lambda_)

    def coefficients(self):
        return self.strength, 0.0


class L2Regularizer(Regularizer):
    name, kind = "L2", RegularizationType.L2

    def __init__(self, lambda_: float = 0.01):
        self.strength = float(lambda_)

    def coefficients(self):
        return 0.0, self.strength


class ElasticNetRegularizer(Regularizer):
    name, kind = "ElasticNet", RegularizationType.ELASTIC_NET

    def __init__(self, lambda_: float = 0.01, l1_ratio: float = 0.5):
        self.strength = float(lambda_)
        self.l1_ratio = float(l1_ratio)

    def coefficients(self):
        return self.strength * self.l1_ratio, self.strength * (1.0 - self.l1_ratio)

    def get_l1_ratio(self) -> float:
        return self.l1_ratio

    def set_l1_ratio(self, r: float) -> None:
        self.l1_ratio = float(r)


class WeightDecayRegularizer(Regularizer):
    name, kind = "WeightDecay", RegularizationType.WEIGHT_DECAY

    def __init__(self, decay_rate: float = 1e-4):
        self.strength = float(decay_rate)

    def coefficients(self):
        return 0.0, self.strength

    def counts_in_loss(self) -> bool:
        return False

    def apply_decay(self, weights: Sequence[torch.Tensor], learning_rate: float) -> None:
        for w in weights:
            w.mul_(1.0 - learning_rate * self.strength)


class AdvancedDropout:
    """Scheduled dropout rate (regularization.cpp:160-185): linear warm-up
    from 0 to `base_rate` over `warmup_epochs`, then (adaptive) x1.1 when
    the validation loss rose >5%, x0.9 (floored at base/2) when it fell
    >5%; clamped to [0, 0.95].  `bind(model)` pushes the rate into every
    Dropout layer of a model (the layers read it at launch time)."""

    def __init__(self, base_rate: float = 0.5, warmup_epochs: int = 10, adaptive: bool = False):
        self.base_rate = float(base_rate)
        self.current_rate = float(base_rate)
        self.warmup_epochs = int(warmup_epochs)
        self.current_epoch = 0
        self.adaptive = bool(adaptive)
        self._prev_loss: Optional[float] = None
        self._layers = []

    def update_rate(self, epoch: int, validation_loss: float = 0.0) -> None:
        self.current_epoch = epoch
        if epoch < self.warmup_epochs:
            self.current_rate = self.base_rate * (epoch / max(self.warmup_epochs, 1))
        elif self.adaptive and validation_loss > 0.0:
            prev = self._prev_loss if self._prev_loss is not None else validation_loss
            if validation_loss > prev * 1.05:
                self.current_rate = min(self.current_rate * 1.1, 0.8)
            elif validation_loss < prev * 0.95:
                self.current_rate = max(self.current_rate * 0.9, self.base_rate * 0.5)
            self._prev_loss = validation_loss
        else:
            self.current_rate = self.base_rate
        self.current_rate = min(max(self.current_rate, 0.0), 0.95)
        for layer in self._layers:
            layer.rate = self.current_rate

    def get_current_rate(self) -> float:
        return self.current_rate

    def bind(self, model) -> "AdvancedDropout":
        from ..models import layers as L

        self._layers = [l for l in model.m_layers if isinstance(l, L.DropoutLayer)]
        for layer in self._layers:
            layer.rate = self.current_rate
        return self

    def apply(self, x: torch.Tensor, training: bool = True) -> torch.Tensor:
        if not training or self.current_rate == 0.0:
            return x
        from ..ops import nn as NN

        return NN.dropout(x, self.current_rate)


class RegularizationManager:
    def __init__(self):
        self.regularizers: List[Regularizer] = []
        self.weights: List[float] = []
        self.enabled = True
        self._loss_dev: Optional[torch.Tensor] = None

    def add_regularizer(self, regularizer: Regularizer, weight: float = 1.0) -> None:
        self.regularizers.append(regularizer)
        self.weights.append(float(weight))

    def set_enabled(self, enabled: bool) -> None:
        self.enabled = bool(enabled)

    def is_enabled(self) -> bool:
        return self.enabled

    def clear(self) -> None:
        self.regularizers.clear()
        self.weights.clear()

    def size(self) -> int:
        return len(self.regularizers)

    __len__ = size

    def combined(self) -> Tuple[float, float, float, float]:
        """(l1, l2) for the gradient and (l1, l2) for the loss."""
        gl1 = gl2 = ll1 = ll2 = 0.0
        for r, w in zip(self.regularizers, self.weights):
            a, b = r.coefficients()
            gl1 += w * a
            gl2 += w * b
            if r.counts_in_loss():
                ll1 += w * a
                ll2 += w * b
        return gl1, gl2, ll1, ll2

    # ---------------------------------------------------------- per-tensor API
    def compute_total_loss(self, weights: Sequence[torch.Tensor]) -> float:
        if not self.enabled:
            return 0.0
        return sum(w * r.compute_loss(weights) for r, w in zip(self.regularizers, self.weights))

    def compute_total_gradients(self, weights: Sequence[torch.Tensor]) -> List[torch.Tensor]:
        out = [torch.zeros_like(w, dtype=torch.float32) for w in weights]
        if not self.enabled:
            return out
        for r, wt in zip(self.regularizers, self.weights):
            for o, g in zip(out, r.compute_gradients(weights)):
                o.add_(wt * g)
        return out

    def get_stats(self, weights: Sequence[torch.Tensor]) -> dict:
        losses = [w * r.compute_loss(weights) for r, w in zip(self.regularizers, self.weights)]
        return {"total_loss": sum(losses), "individual_losses": losses,
                "regularizer_names": [r.name for r in self.regularizers]}

    # ---------------------------------------------------------- fused model path
    @staticmethod
    def _decay_runs(store) -> List[Tuple[int, int]]:
        """Contiguous [start, end) runs of decayed parameters, merged across
        the zero padding between them (zero weights add zero penalty)."""
        from ..models.params import ALIGN_ELEMS, _round_up

        runs: List[Tuple[int, int]] = []
        for p in sorted(store.params, key=lambda q: q.offset):
            if not p.decay:
                continue
            a, b = p.offset, min(store.numel, p.offset + _round_up(p.numel, ALIGN_ELEMS))
            if runs and runs[-1][1] == a:
                runs[-1] = (runs[-1][0], b)
            else:
                runs.append((a, b))
        return runs

    def loss_buffer(self, device) -> torch.Tensor:
        if self._loss_dev is None or self._loss_dev.device != torch.device(device):
            self._loss_dev = torch.zeros(1, dtype=torch.float32, device=device)
        return self._loss_dev

    def apply_to_store(self, store, grad_scale: Optional[torch.Tensor] = None,
                       track_loss: bool = True) -> Optional[torch.Tensor]:
        """Add the penalty gradients of every decayed parameter to the flat
        gradient (and the penalty value to a device scalar, returned)."""
        if not self.enabled or not self.regularizers:
            return None
        gl1, gl2, ll1, ll2 = self.combined()
        loss = self.loss_buffer(store.device) if track_loss else None
        if loss is not None:
            loss.zero_()
        cuda = store.device.type == "cuda"
        for a, b in self._decay_runs(store):
            w = store.master[a:b]
            g = store.grad[a:b]
            if cuda:
                K.N().regularize(w, g, gl1, gl2, ll1, ll2, loss, grad_scale)
            else:
                k = float(grad_scale) if grad_scale is not None else 1.0
                g.add_(k * (gl1 * torch.sign(w) + gl2 * w))
                if loss is not None:
                    loss.add_(ll1 * w.abs().sum() + 0.5 * ll2 * (w * w).sum())
        return loss


# regularization_factory (regularization.h:230-250)
def create_l2_regularization(lambda_: float = 0.01) -> RegularizationManager:
    m = RegularizationManager()
    m.add_regularizer(L2Regularizer(lambda_))
    return m


def create_elastic_net(lambda_: float = 0.01, l1_ratio: float = 0.5) -> RegularizationManager:
    m = RegularizationManager()
    m.add_regularizer(ElasticNetRegularizer(lambda_, l1_ratio))
    return m


def create_weight_decay(decay_rate: float = 1e-4) -> RegularizationManager:
    m = RegularizationManager()
    m.add_regularizer(WeightDecayRegularizer(decay_rate))
    return m


def create_comprehensive_regularization(l2_lambda: float = 0.01, weight_decay: float = 1e-4,
                                        include_l1: bool = False, l1_lambda: float = 0.001) -> RegularizationManager:
    m = RegularizationManager()
    m.add_regularizer(L2Regularizer(l2_lambda))
    m.add_regularizer(WeightDecayRegularizer(weight_decay))
    if include_l1:
        m.add_regularizer(L1Regularizer(l1_lambda))
    return m
