"""Mixed precision (include/dlvk/training/mixed_precision.h:15-190,
src/training/mixed_precision.cpp).

PrecisionMode.FP16 / MIXED map to bf16 compute with fp32 master weights:
Blackwell's tensor cores take bf16 at the fp16 rate and bf16 has fp32's
exponent range, so the compute dtype of a model built under MIXED is bf16
(the reference's FP16 mode converted tensors on the host and left compute
in fp32).

`GradientScaler` is dynamic loss scaling kept entirely on the device, so a
captured training-step graph replays it:

* `scale` (fp32[1]), `good_steps` (int32[1]) and `found_inf` (int32[1])
  are device tensors;
* `scale_grad_output(dout)` multiplies the loss gradient by `scale`
  (one kernel reading the scale from memory);
* `unscale_gradients(optimizer, store)` runs one statistics pass over the
  flat gradient (non-finite flag + the optimizer's clip coefficient at the
  unscaled norm); the optimizer's device hyper block points its
  `skip_flag_ptr` at `found_inf` and its `grad_scale` holds 1/scale, so the
  optimizer kernel unscales as it updates and skips a step with inf/nan;
* `update()` grows the scale x`growth_factor` after `scale_window` clean
  steps, backs off x`backoff_factor` on overflow, and writes the new 1/scale
  into every attached hyper block.

Semantics follow mixed_precision.h:25-60 (init 2^16, window 2000, backoff
0.5, growth 2).
"""
from __future__ import annotations

import enum
import threading
from typing import Callable, List, Optional

import torch

from ..ops import core as K
from ..ops.optim_kernels import field_offset, set_field


class PrecisionMode(enum.Enum):
    FP32 = 0
    FP16 = 1
    MIXED = 2

    @property
    def compute_dtype(self) -> torch.dtype:
        return torch.float32 if self is PrecisionMode.FP32 else torch.bfloat16


class GradientScaler:
    def __init__(self, init_scale: float = 65536.0, scale_factor: float = 2.0, scale_window: int = 2000,
                 backoff_factor: float = 0.5, growth_factor: float = 2.0, enabled: bool = True, device=None,
                 min_scale: float = 1.0, max_scale: float = 65536.0):
        self.scale_factor = float(scale_factor)
        self.scale_window = int(scale_window)
        self.backoff_factor = float(backoff_factor)
        self.growth_factor = float(growth_factor)
        self.min_scale, self.max_scale = float(min_scale), float(max_scale)
        self.enabled = bool(enabled)
        dev = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self.device = dev
        self.scale = torch.full((1,), float(init_scale), dtype=torch.float32, device=dev)
        self.inv_scale = torch.full((1,), 1.0 / float(init_scale), dtype=torch.float32, device=dev)
        self.good_steps = torch.zeros(1, dtype=torch.int32, device=dev)
        self.found_inf = torch.zeros(1, dtype=torch.int32, device=dev)
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
        self._scratch = None
        self._hyper_views: List[torch.Tensor] = []
        self.skipped_steps = 0

    # ------------------------------------------------------------------ API
    def get_scale(self) -> float:
        return float(self.scale) if self.enabled else 1.0

    def set_enabled(self, enabled: bool) -> None:
        self.enabled = bool(enabled)

    def is_enabled(self) -> bool:
        return self.enabled

    def has_overflow(self) -> bool:
        return bool(int(self.found_inf))

    @property
    def _cuda(self) -> bool:
        return self.device.type == "cuda"

    def attach(self, optimizer, store) -> None:
        """Point `optimizer`'s device hyper block for `store` at this scaler."""
        st = optimizer.state(store)
        optimizer._scaler = self
        if st.hyper is None:
            return  # CPU: the optimizer reads inv_scale and found_inf from the scaler
        view = st.hyper[field_offset("grad_scale"):field_offset("grad_scale") + 4].view(torch.float32)
        if not any(v.data_ptr() == view.data_ptr() for v in self._hyper_views):
            view.copy_(self.inv_scale)
            set_field(st.hyper, "skip_flag_ptr", self.found_inf.data_ptr())
            self._hyper_views.append(view)
        optimizer._scaler = self

    def detach(self, optimizer, store) -> None:
        st = optimizer.state(store)
        if st.hyper is not None:
            set_field(st.hyper, "skip_flag_ptr", 0)
            set_field(st.hyper, "grad_scale", 1.0)
        optimizer._scaler = None

    def scale_loss(self, loss: torch.Tensor) -> torch.Tensor:
        """loss * scale (a new tensor)."""
        if not self.enabled:
            return loss
        out = loss.detach().clone().contiguous()
        return self.scale_grad_output(out)

    def scale_grad_output(self, dout: torch.Tensor) -> torch.Tensor:
        """In place: dout *= scale (the gradient of the scaled loss)."""
        if not self.enabled:
            return dout
        if self._cuda:
            K.N().scale_by_device_scalar(dout, self.scale)
        else:
            dout.mul_(self.scale.to(dout.dtype))
        return dout

    def unscale_gradients(self, optimizer, store=None) -> None:
        """Non-finite check (and clip coefficient) of the scaled gradients.
        The division by the scale happens inside the optimizer update."""
        if not self.enabled:
            return
        if store is None:
            store = next(iter(optimizer._states.values())).store
        self.attach(optimizer, store)
        g = store.grad
        st = optimizer.state(store)
        max_norm = float(optimizer.clip_norm) if optimizer.clip_norm is not None else 0.0
        if self._cuda:
            if self._scratch is None:
                self._scratch = torch.empty(K.N().grad_stats_scratch_floats(), device=self.device)
            K.N().grad_stats(g, 1.0, max_norm, self._sumsq, self.found_inf, st.clip if max_norm > 0 else None,
                             False, self._scratch, scale_dev=self.inv_scale)
        else:
            bad = not bool(torch.isfinite(g).all())
            self.found_inf.fill_(int(bad))
            gu = g.float() * self.inv_scale
            if max_norm > 0:
                st.clip.fill_(min(1.0, max_norm / (float(gu.norm()) + 1e-6)))

    def update(self) -> None:
        if not self.enabled:
            return
        if self._cuda:
            K.N().scaler_update(self.scale, self.good_steps, self.found_inf, self.growth_factor,
                                self.backoff_factor, self.scale_window, self.min_scale, self.max_scale,
                                self.inv_scale)
            for v in self._hyper_views:
                v.copy_(self.inv_scale)
        else:
            if int(self.found_inf):
                self.scale.mul_(self.backoff_factor).clamp_(min=self.min_scale)
                self.good_steps.zero_()
                self.skipped_steps += 1
            else:
                self.good_steps += 1
                if int(self.good_steps) >= self.scale_window:
                    self.scale.mul_(self.growth_factor).clamp_(max=self.max_scale)
                    self.good_steps.zero_()
            self.inv_scale.copy_(1.0 / self.scale)

    def state_dict(self) -> dict:
        return {"scale": float(self.scale), "good_steps": int(self.good_steps)}

    def load_state_dict(self, d: dict) -> None:
        self.scale.fill_(float(d["scale"]))
        self.inv_scale.fill_(1.0 / float(d["scale"]))
        self.good_steps.fill_(int(d.get("good_steps", 0)))
        for v in self._hyper_views:
            v.copy_(self.inv_scale)


class MixedPrecisionContext:
    def __init__(self, mode: PrecisionMode = PrecisionMode.MIXED, enable_scaler: bool = True,
                 autocast: bool = True, device=None):
        self.mode = mode
        self.autocast_enabled = autocast
        self.scaler = GradientScaler(device=device) if (enable_scaler and mode is not PrecisionMode.FP32) else None

    def get_mode(self) -> PrecisionMode:
        return self.mode

    def get_scaler(self) -> Optional[GradientScaler]:
        return self.scaler

    def is_autocast_enabled(self) -> bool:
        return self.autocast_enabled

    def to_forward_precision(self, x: torch.Tensor) -> torch.Tensor:
        want = self.mode.compute_dtype
        if not x.is_floating_point() or x.dtype == want:
            return x
        if x.is_cuda:
            return K.unary(x.contiguous(), K.UN_COPY, out_dtype=want)
        return x.to(want)

    def to_backward_precision(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_floating_point() or x.dtype == torch.float32:
            return x
        if x.is_cuda:
            return K.unary(x.contiguous(), K.UN_COPY, out_dtype=torch.float32)
        return x.float()

    def estimate_memory_savings(self) -> float:
        """Fraction of activation/weight-copy bytes saved versus fp32."""
        return 0.0 if self.mode is PrecisionMode.FP32 else 0.5


class _AutocastState(threading.local):
    enabled = False
    mode = PrecisionMode.FP32


_autocast = _AutocastState()


class AutocastContext:
    """Thread-local autocast scope; models built inside it pick the mode's
    compute dtype (`Sequential(dtype="auto")`)."""

    def __init__(self, enabled: bool, mode: PrecisionMode = PrecisionMode.FP16):
        self.enabled, self.mode = bool(enabled), mode

    def __enter__(self):
        self._prev = (_autocast.enabled, _autocast.mode)
        _autocast.enabled, _autocast.mode = self.enabled, self.mode
        return self

    def __exit__(self, *exc):
        _autocast.enabled, _autocast.mode = self._prev
        return False

    @staticmethod
    def is_enabled() -> bool:
        return _autocast.enabled

    @staticmethod
    def get_mode() -> PrecisionMode:
        return _autocast.mode


def autocast_dtype(default: torch.dtype) -> torch.dtype:
    return _autocast.mode.compute_dtype if _autocast.enabled else default


class MixedPrecisionTrainer:
    def __init__(self, mode: PrecisionMode = PrecisionMode.MIXED, device=None):
        self.context = MixedPrecisionContext(mode, device=device)

    def get_context(self) -> MixedPrecisionContext:
        return self.context

    def forward_with_autocast(self, forward_fn: Callable[[], torch.Tensor]) -> torch.Tensor:
        with AutocastContext(self.context.is_autocast_enabled(), self.context.mode):
            return forward_fn()

    def backward_with_scaling(self, model, dout: torch.Tensor, optimizer) -> None:
        """Backward of the scaled loss gradient, overflow check, optimizer
        step (skipped on overflow) and scale update."""
        sc = self.context.scaler
        if sc is not None:
            sc.scale_grad_output(dout)
        model.backward(dout)
        if sc is not None:
            sc.unscale_gradients(optimizer, model.store)
        optimizer.step(model)
        if sc is not None:
            sc.update()

    def get_memory_stats(self, model) -> dict:
        n = model.parameter_count()
        fp32 = 4 * n
        mixed = fp32 + (2 * n if self.context.mode is not PrecisionMode.FP32 else 0)
        return {"fp32_memory": fp32, "fp16_memory": 2 * n,
                "savings_ratio": self.context.estimate_memory_savings(), "total_param_bytes": mixed}
