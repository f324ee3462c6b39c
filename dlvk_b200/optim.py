"""Optimizers (include/dlvk/optimizers/optimizers.h:11-155): SGD (with
momentum), Adam and RMSprop, plus the learning-rate schedulers of
include/dlvk/optimizers/lr_scheduler.h and `GradientClipping`.

On the GPU an optimizer keeps its state (m, v / momentum / square average)
as flat fp32 buffers parallel to the model's ParamStore and updates every
parameter with ONE kernel launch (optim.cu), reading its hyper-parameters
from a small device block so a captured CUDA graph can replay many steps.
Adam applies the bias corrections 1/(1-beta^t) that the reference shader
documents (shaders/adam_update.comp:27-28) but its host code disabled
(src/tensor/tensor_ops.cpp:2353-2354); `bias_correction=False` restores the
reference behaviour.  The step counter advances once per `step()` (the
reference counted it twice, src/optimizers/adam.cpp:18,37).
"""
from __future__ import annotations

import math
from typing import Dict, Iterable, List, Optional

import torch

from .ops import core as K
from .ops.optim_kernels import make_hyper, set_field, read_hyper


class _State:
    def __init__(self, store, kind, opt):
        dev = store.device
        self.store = store
        self.cuda = dev.type == "cuda"
        n = store.numel
        self.m = torch.zeros(n, dtype=torch.float32, device=dev) if kind in (K.OPT_ADAM, K.OPT_SGD) else None
        self.v = torch.zeros(n, dtype=torch.float32, device=dev) if kind in (K.OPT_ADAM, K.OPT_RMSPROP) else None
        self.clip = torch.ones(1, dtype=torch.float32, device=dev)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self.scratch = None
        self.step = 0
        if self.cuda:
            self.hyper = make_hyper(dev, lr=opt.lr, beta1=opt.beta1, beta2=opt.beta2, eps=opt.eps,
                                    weight_decay=opt.weight_decay, momentum=opt.momentum, alpha=opt.alpha,
                                    grad_scale=1.0, bias_correction=opt.bias_correction,
                                    decoupled_wd=opt.decoupled_wd)
        else:
            self.hyper = None


class Optimizer:
    kind = K.OPT_SGD

    def __init__(self, learning_rate: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999, epsilon: float = 1e-8,
                 momentum: float = 0.0, alpha: float = 0.99, weight_decay: float = 0.0, bias_correction: bool = True,
                 decoupled_wd: bool = False):
        self.lr = float(learning_rate)
        self.beta1, self.beta2, self.eps = float(beta1), float(beta2), float(epsilon)
        self.momentum, self.alpha = float(momentum), float(alpha)
        self.weight_decay = float(weight_decay)
        self.bias_correction = bool(bias_correction)
        self.decoupled_wd = bool(decoupled_wd)
        self.clip_norm: Optional[float] = None
        self.clip_value: Optional[float] = None
        self.clip_range: Optional[tuple] = None  # (min, max) from set_grad_clip_value
        self._states: Dict[int, _State] = {}
        self._tensor_stores: Dict[tuple, "_TensorStore"] = {}
        self._scaler = None  # a GradientScaler attached to this optimizer's hyper blocks

    # ---------------------------------------------------------------- API
    def get_learning_rate(self) -> float:
        return self.lr

    def set_learning_rate(self, lr: float) -> None:
        self.lr = float(lr)
        for st in self._states.values():
            if st.hyper is not None:
                set_field(st.hyper, "lr", self.lr)

    def set_gradient_clipping(self, max_norm: Optional[float] = None, clip_value: Optional[float] = None) -> None:
        """Clip by global norm (per optimizer step) and/or by value."""
        self.clip_norm = max_norm
        self.clip_value = clip_value
        self.clip_range = None

    # Reference spellings (include/dlvk/optimizers/optimizers.h:20-45).
    def set_lr(self, lr: float) -> None:
        self.set_learning_rate(lr)

    def get_lr(self) -> float:
        return self.lr

    def set_grad_clip_norm(self, max_norm: float) -> None:
        """Scale the gradients of each update by min(1, max_norm / ||g||)."""
        self.clip_norm = float(max_norm)

    def set_grad_clip_value(self, min_val: float, max_val: float) -> None:
        """Clamp every gradient element to [min_val, max_val] before the update."""
        if float(min_val) > float(max_val):
            raise ValueError(f"clip range [{min_val}, {max_val}] is empty")
        self.clip_value = None
        self.clip_range = (float(min_val), float(max_val))

    def disable_grad_clipping(self) -> None:
        self.clip_norm = self.clip_value = self.clip_range = None

    def _clip_bounds(self) -> Optional[tuple]:
        if self.clip_range is not None:
            return self.clip_range
        if self.clip_value is not None:
            return (-self.clip_value, self.clip_value)
        return None

    def zero_gradients(self) -> None:
        """Zero the gradient buffers of every store and tensor this optimizer
        has updated, and mark the packed parameters so the next backward
        overwrites instead of accumulating."""
        for st in self._states.values():
            zero = getattr(st.store, "zero_grad", None)
            if zero is not None:
                zero(set_to_zero=True)
            elif st.store.grad is not None:
                st.store.grad.zero_()

    def update_parameter(self, parameter: torch.Tensor, gradient: torch.Tensor) -> None:
        """Apply one update of this optimizer's rule to a standalone tensor
        in place (reference Optimizer::update_parameter,
        include/dlvk/optimizers/optimizers.h:24-25).  The optimizer state
        (momentum, m / v, step count) is kept per tensor storage, so
        repeated calls on the same tensor continue one trajectory.  An
        fp32 master copy is kept for a bf16 / fp16 tensor, which receives
        the rounded result.  The gradient is not modified."""
        from .tensor import Tensor as FacadeTensor

        if isinstance(parameter, FacadeTensor):
            parameter = parameter.data
        if isinstance(gradient, FacadeTensor):
            gradient = gradient.data
        if not parameter.is_contiguous():
            raise ValueError("update_parameter needs a contiguous parameter tensor")
        if gradient.numel() != parameter.numel():
            raise ValueError(f"gradient has {gradient.numel()} elements, parameter {parameter.numel()}")
        key = (parameter.data_ptr(), parameter.numel(), parameter.dtype, str(parameter.device))
        ts = self._tensor_stores.get(key)
        if ts is None:
            ts = _TensorStore(parameter)
            self._tensor_stores[key] = ts
        ts.grad = gradient.detach().reshape(-1).to(parameter.device, torch.float32, copy=True)
        self.step(ts)
        ts.grad = None

    def state(self, store) -> _State:
        st = self._states.get(id(store))
        if st is None:
            st = _State(store, self.kind, self)
            self._states[id(store)] = st
            if st.hyper is not None:
                set_field(st.hyper, "clip_coef_ptr", st.clip.data_ptr())
        return st

    def advance(self, store) -> None:
        """Advance the step counter (and bias corrections) for `store`."""
        st = self.state(store)
        if st.cuda:
            st.step += 1  # host mirror; the device counter skips overflowed steps
            K.N().optim_advance(st.hyper)
        elif not self._cpu_skip():
            st.step += 1

    def prepare_grads(self, store) -> None:
        """Global-norm clipping coefficient and value clipping (device side)."""
        st = self.state(store)
        scaled = self._scaler is not None and self._scaler.enabled
        if scaled and self._clip_bounds() is not None:
            raise ValueError("value clipping is not defined on loss-scaled gradients; use clip_norm")
        if scaled:
            return  # the scaler computed the overflow flag and the clip coefficient
        bounds = self._clip_bounds()
        if bounds is not None:
            g = store.grad
            if st.cuda:
                K.N().unary(g, K.UN_CLAMP, bounds[0], bounds[1], out=g)
            else:
                g.clamp_(bounds[0], bounds[1])
        if self.clip_norm is not None:
            if st.cuda:
                if st.scratch is None:
                    st.scratch = torch.empty(K.N().grad_stats_scratch_floats(), device=store.device)
                K.N().grad_stats(store.grad, 1.0, float(self.clip_norm), st.sumsq, st.flag, st.clip, False,
                                 st.scratch)
            else:
                norm = float(store.grad.norm())
                st.clip.fill_(min(1.0, self.clip_norm / (norm + 1e-6)))

    def update_range(self, store, start: int, end: int, grad: Optional[torch.Tensor] = None,
                     extra_scale: float = 1.0, max_ctas: int = 0) -> None:
        """Apply the update to flat elements [start, end); `max_ctas` caps
        the kernel's grid (an update running beside other kernels)."""
        st = self.state(store)
        g = store.grad[start:end] if grad is None else grad
        p = store.master[start:end]
        m = st.m[start:end] if st.m is not None else None
        v = st.v[start:end] if st.v is not None else None
        pb = store.value[start:end] if store.value is not store.master else None
        if st.cuda:
            K.N().optim_update(self.kind, st.hyper, p, g, m, v, pb, extra_scale, max_ctas)
        else:
            if self._cpu_skip():
                return
            if self._scaler is not None and self._scaler.enabled:
                extra_scale = extra_scale * float(self._scaler.inv_scale)
            self._cpu_update(st, p, g.float() * extra_scale * float(st.clip), m, v)
            if pb is not None:
                pb.copy_(p)

    def step(self, model_or_store) -> None:
        store = getattr(model_or_store, "store", model_or_store)
        self.advance(store)
        self.prepare_grads(store)
        self.update_range(store, 0, store.numel)

    def update_parameters(self, params: Iterable) -> None:
        """Update just these parameters (reference Layer::update_parameters)."""
        params = list(params)
        by_store = {}
        for p in params:
            by_store.setdefault(id(p.store), (p.store, []))[1].append(p)
        for store, ps in by_store.values():
            self.advance(store)
            self.prepare_grads(store)
            for p in ps:
                self.update_range(store, p.offset, p.offset + p.numel)

    def _cpu_skip(self) -> bool:
        sc = self._scaler
        return sc is not None and sc.enabled and bool(int(sc.found_inf))

    # ---------------------------------------------------------------- CPU reference update
    def _cpu_update(self, st, p, g, m, v):
        lr = self.lr
        if self.weight_decay and not self.decoupled_wd:
            g = g + self.weight_decay * p
        t = st.step
        if self.kind == K.OPT_ADAM:
            m.mul_(self.beta1).add_((1 - self.beta1) * g)
            v.mul_(self.beta2).add_((1 - self.beta2) * g * g)
            bc1 = 1.0 / (1 - self.beta1 ** t) if self.bias_correction else 1.0
            bc2 = 1.0 / (1 - self.beta2 ** t) if self.bias_correction else 1.0
            if self.weight_decay and self.decoupled_wd:
                p.mul_(1 - lr * self.weight_decay)
            p.sub_(lr * (m * bc1) / (torch.sqrt(v * bc2) + self.eps))
        elif self.kind == K.OPT_SGD:
            if self.momentum:
                m.mul_(self.momentum).add_(g)
                p.sub_(lr * m)
            else:
                p.sub_(lr * g)
        else:
            v.mul_(self.alpha).add_((1 - self.alpha) * g * g)
            p.sub_(lr * g / (torch.sqrt(v) + self.eps))

    # ---------------------------------------------------------------- checkpoint state
    def state_tensors(self, store) -> List:
        st = self.state(store)
        out = []
        if st.m is not None:
            out.append(("optim.m", st.m))
        if st.v is not None:
            out.append(("optim.v", st.v))
        return out

    def state_meta(self, store) -> dict:
        st = self.state(store)
        step = int(read_hyper(st.hyper)["step"]) if st.hyper is not None else st.step
        return {"type": type(self).__name__, "step": step, "lr": self.lr, "beta1": self.beta1,
                "beta2": self.beta2, "eps": self.eps, "momentum": self.momentum, "alpha": self.alpha,
                "weight_decay": self.weight_decay, "bias_correction": self.bias_correction}

    def load_state_meta(self, store, meta: dict) -> None:
        st = self.state(store)
        st.step = int(meta.get("step", 0))
        self.set_learning_rate(float(meta.get("lr", self.lr)))
        if st.hyper is not None:
            set_field(st.hyper, "step", st.step)
            if self.bias_correction and st.step > 0:
                set_field(st.hyper, "bc1", 1.0 / (1 - self.beta1 ** st.step))
                set_field(st.hyper, "bc2", 1.0 / (1 - self.beta2 ** st.step))


class _TensorStore:
    """A one-tensor stand-in for a ParamStore, used by update_parameter:
    `master` is the fp32 flat view being updated (the tensor itself when it
    is fp32), `value` the caller's lower-precision tensor when there is one."""

    def __init__(self, parameter: torch.Tensor):
        self.device = parameter.device
        self.numel = parameter.numel()
        flat = parameter.detach().view(-1)
        if parameter.dtype == torch.float32:
            self.master = self.value = flat
        else:
            self.master = flat.float()
            self.value = flat
        self.grad = None


class SGD(Optimizer):
    """v = mu v + g; p -= lr v (src/optimizers/sgd.cpp:55-76)."""

    kind = K.OPT_SGD

    def __init__(self, learning_rate: float = 0.01, momentum: float = 0.0, weight_decay: float = 0.0):
        super().__init__(learning_rate, momentum=momentum, weight_decay=weight_decay)


class Adam(Optimizer):
    kind = K.OPT_ADAM

    def __init__(self, learning_rate: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999,
                 epsilon: float = 1e-8, weight_decay: float = 0.0, bias_correction: bool = True,
                 decoupled_wd: bool = False):
        super().__init__(learning_rate, beta1, beta2, epsilon, weight_decay=weight_decay,
                         bias_correction=bias_correction, decoupled_wd=decoupled_wd)


class RMSprop(Optimizer):
    """sq = a sq + (1 - a) g^2; p -= lr g / (sqrt(sq) + eps)
    (declared in include/dlvk/optimizers/optimizers.h:107-141)."""

    kind = K.OPT_RMSPROP

    def __init__(self, learning_rate: float = 1e-3, alpha: float = 0.99, epsilon: float = 1e-8,
                 weight_decay: float = 0.0):
        super().__init__(learning_rate, epsilon=epsilon, alpha=alpha, weight_decay=weight_decay)


class GradientClipping:
    """Global-norm utilities (src/optimizers/optimizers.cpp:9-55)."""

    @staticmethod
    def compute_grad_norm(grads: Iterable[torch.Tensor]) -> float:
        tot = 0.0
        for g in grads:
            tot += float(K.reduce(g, K.RED_SUMSQ))
        return math.sqrt(tot)

    @staticmethod
    def clip_grad_norm(grads: List[torch.Tensor], max_norm: float) -> float:
        norm = GradientClipping.compute_grad_norm(grads)
        if norm > max_norm:
            s = max_norm / (norm + 1e-6)
            for g in grads:
                if g.is_cuda:
                    K.N().unary(g, K.UN_SCALE, s, 0.0, out=g)
                else:
                    g.mul_(s)
        return norm

    @staticmethod
    def clip_grad_value(grads: List[torch.Tensor], clip_value: float) -> None:
        for g in grads:
            if g.is_cuda:
                K.N().unary(g, K.UN_CLAMP, -clip_value, clip_value, out=g)
            else:
                g.clamp_(-clip_value, clip_value)


# ------------------------------------------------------------------ LR schedulers
class LRScheduler:
    """get_lr(step, base_lr) (include/dlvk/optimizers/lr_scheduler.h:7-71)."""

    def get_lr(self, step: int, base_lr: float) -> float:  # pragma: no cover - abstract
        raise NotImplementedError

    def apply(self, optimizer: Optimizer, step: int, base_lr: float) -> float:
        lr = self.get_lr(step, base_lr)
        optimizer.set_learning_rate(lr)
        return lr


class StepLRScheduler(LRScheduler):
    def __init__(self, step_size: int, gamma: float = 0.1):
        self.step_size, self.gamma = int(step_size), float(gamma)

    def get_lr(self, step, base_lr):
        return base_lr * self.gamma ** (step // self.step_size)


class ExponentialLRScheduler(LRScheduler):
    def __init__(self, gamma: float):
        self.gamma = float(gamma)

    def get_lr(self, step, base_lr):
        return base_lr * self.gamma ** step


class CosineAnnealingLRScheduler(LRScheduler):
    def __init__(self, T_max: int, eta_min: float = 0.0):
        self.T_max, self.eta_min = int(T_max), float(eta_min)

    def get_lr(self, step, base_lr):
        return self.eta_min + (base_lr - self.eta_min) * (1 + math.cos(math.pi * (step % (self.T_max + 1)) / self.T_max)) / 2


class LinearLRScheduler(LRScheduler):
    def __init__(self, start_factor: float = 1.0, end_factor: float = 0.0, total_steps: int = 100):
        self.start, self.end, self.total = float(start_factor), float(end_factor), int(total_steps)

    def get_lr(self, step, base_lr):
        f = self.start + (self.end - self.start) * min(step, self.total) / max(1, self.total)
        return base_lr * f
