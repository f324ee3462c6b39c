"""Loss functions (include/dlvk/loss/loss_functions.h:8-51,
src/loss/loss_functions.cpp).

`forward(pred, target)` / `backward(pred, target)` keep the reference
semantics on probabilities:
  CrossEntropyLoss       -sum t log(p + 1e-8) / B                    (:127-135)
  MeanSquaredError       mean((p - t)^2), grad 2 (p - t) / N           (:59-64)
  BinaryCrossEntropyLoss clamp eps 1e-7, mean, grad (p-t)/(p(1-p))/N   (:189-238)
CrossEntropyLoss.backward returns -t / (p + 1e-8) / B, the gradient w.r.t.
the softmax output, which the standard softmax Jacobian turns into the
(p - t) / B logits gradient the reference obtained with an identity softmax
backward.  Training uses `value_and_grad(..., from_logits=True)`: one fused
softmax + cross-entropy kernel producing the loss and dlogits together.
Targets may be int class ids or one-hot / probability rows.
"""
from __future__ import annotations

import torch

from .ops import core as K
from .ops import functional as Fn


def _to_probs(target: torch.Tensor, cols: int) -> torch.Tensor:
    if target.is_floating_point():
        return target.float()
    t = torch.zeros(target.numel(), cols, dtype=torch.float32, device=target.device)
    t[torch.arange(target.numel(), device=target.device), target.reshape(-1).long()] = 1.0
    return t


def _unwrap(x):
    from .tensor import Tensor as FacadeTensor

    return x.data if isinstance(x, FacadeTensor) else x


class LossFunction:
    fuses_softmax = False

    def forward(self, predictions, targets):
        raise NotImplementedError

    def backward(self, predictions, targets):
        raise NotImplementedError

    def value_and_grad(self, out, target, from_logits: bool = False):
        raise NotImplementedError

    __call__ = lambda self, p, t: self.forward(p, t)  # noqa: E731


class CrossEntropyLoss(LossFunction):
    fuses_softmax = True

    def forward(self, predictions, targets):
        p = _unwrap(predictions).float()
        p2 = p.reshape(-1, p.shape[-1])
        t = _to_probs(_unwrap(targets).to(p.device), p2.shape[1]).reshape(p2.shape)
        return -(t * torch.log(p2 + 1e-8)).sum() / p2.shape[0]

    def backward(self, predictions, targets):
        p = _unwrap(predictions)
        p2 = p.reshape(-1, p.shape[-1]).float()
        t = _to_probs(_unwrap(targets).to(p.device), p2.shape[1]).reshape(p2.shape)
        return (-t / (p2 + 1e-8) / p2.shape[0]).to(p.dtype).reshape(p.shape)

    def value_and_grad(self, out, target, from_logits: bool = False):
        out = _unwrap(out)
        target = _unwrap(target)
        rows = out.numel() // out.shape[-1]
        if from_logits:
            tgt = target.to(out.device)
            if not tgt.is_floating_point():
                tgt = tgt.to(torch.int32)
            loss, dl = Fn.softmax_cross_entropy(out.reshape(rows, out.shape[-1]), tgt.reshape(rows, -1)
                                                if tgt.is_floating_point() else tgt.reshape(rows),
                                                1.0 / rows)
            return loss, dl.reshape(out.shape)
        return self.forward(out, target), self.backward(out, target)


class MeanSquaredError(LossFunction):
    def forward(self, predictions, targets):
        p = _unwrap(predictions)
        loss, _ = K.pointwise_loss(p, _unwrap(targets).to(p.device), K.LOSS_MSE, 1.0 / p.numel(), 0.0, False)
        return loss

    def backward(self, predictions, targets):
        p = _unwrap(predictions)
        _, g = K.pointwise_loss(p, _unwrap(targets).to(p.device), K.LOSS_MSE, 1.0 / p.numel(), 1.0 / p.numel(), True)
        return g

    def value_and_grad(self, out, target, from_logits: bool = False):
        out = _unwrap(out)
        n = out.numel()
        return K.pointwise_loss(out, _unwrap(target).to(out.device), K.LOSS_MSE, 1.0 / n, 1.0 / n, True)


class BinaryCrossEntropyLoss(LossFunction):
    def forward(self, predictions, targets):
        p = _unwrap(predictions)
        loss, _ = K.pointwise_loss(p, _unwrap(targets).to(p.device), K.LOSS_BCE, 1.0 / p.numel(), 0.0, False)
        return loss

    def backward(self, predictions, targets):
        p = _unwrap(predictions)
        _, g = K.pointwise_loss(p, _unwrap(targets).to(p.device), K.LOSS_BCE, 1.0 / p.numel(), 1.0 / p.numel(), True)
        return g

    def value_and_grad(self, out, target, from_logits: bool = False):
        out = _unwrap(out)
        n = out.numel()
        return K.pointwise_loss(out, _unwrap(target).to(out.device), K.LOSS_BCE, 1.0 / n, 1.0 / n, True)


# Reference spellings.
MSELoss = MeanSquaredError
BCELoss = BinaryCrossEntropyLoss


class LossOpsGPU:
    """The reference's per-op loss entry points (include/dlvk/loss/loss_ops_gpu.h:10-60)
    over this library's loss kernels (softmax_loss.cu `pointwise_loss`;
    cross-entropy on probabilities as CrossEntropyLoss).  Each method returns
    its result tensor; the reference wrote it through an out-parameter and
    returned a success flag.  The semantics are the reference's CPU ones:

      mse_forward                    mean((p - t)^2)
      mse_backward                   2 (p - t) / N
      cross_entropy_forward          -sum t log(p + 1e-8) / B    (p: probabilities)
      cross_entropy_backward         -t / (p + 1e-8) / B
      binary_cross_entropy_forward   mean of -(t log p + (1 - t) log(1 - p)), p clamped to [eps, 1 - eps]
      binary_cross_entropy_backward  (p - t) / (p (1 - p)) / N with the same clamp

    The kernels clamp BCE probabilities at 1e-7; a larger `epsilon` clamps
    the predictions first, a smaller one is rejected."""

    def __init__(self, device=None):
        self.device = device

    def initialize(self) -> bool:
        return True

    def mse_forward(self, predictions, targets):
        return MeanSquaredError().forward(predictions, targets)

    def mse_backward(self, predictions, targets):
        return MeanSquaredError().backward(predictions, targets)

    def cross_entropy_forward(self, predictions, targets):
        return CrossEntropyLoss().forward(predictions, targets)

    def cross_entropy_backward(self, predictions, targets):
        return CrossEntropyLoss().backward(predictions, targets)

    @staticmethod
    def _clamped(predictions, epsilon: float):
        p = _unwrap(predictions)
        if epsilon < 1e-7:
            raise ValueError(f"epsilon {epsilon} is below the kernel's 1e-7 probability clamp")
        if epsilon > 1e-7:
            p = K.unary(p, K.UN_CLAMP, float(epsilon), 1.0 - float(epsilon))
        return p

    def binary_cross_entropy_forward(self, predictions, targets, epsilon: float = 1e-7):
        return BinaryCrossEntropyLoss().forward(self._clamped(predictions, epsilon), targets)

    def binary_cross_entropy_backward(self, predictions, targets, epsilon: float = 1e-7):
        return BinaryCrossEntropyLoss().backward(self._clamped(predictions, epsilon), targets)
