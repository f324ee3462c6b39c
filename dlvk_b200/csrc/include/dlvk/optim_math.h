// Per-element optimizer update rule shared by the standalone optimizer kernel
// and the fused all-reduce + optimizer kernel.
#pragma once
#include "dlvk/kernels.h"

namespace dlvk {

// w: parameter (in/out), g: already-scaled gradient, m/v: state (in/out).
__device__ __forceinline__ void opt_apply(int kind, const OptimHyper& h, float& w, float g, float& m, float& v) {
  if (h.weight_decay != 0.f && !h.decoupled_wd) g += h.weight_decay * w;
  if (kind == OPT_ADAM) {
    m = h.beta1 * m + (1.f - h.beta1) * g;
    v = h.beta2 * v + (1.f - h.beta2) * g * g;
    if (h.weight_decay != 0.f && h.decoupled_wd) w -= h.lr * h.weight_decay * w;
    w -= h.lr * (m * h.bc1) / (sqrtf(v * h.bc2) + h.eps);
  } else if (kind == OPT_SGD) {
    if (h.momentum != 0.f) {
      m = h.momentum * m + g;
      w -= h.lr * m;
    } else {
      w -= h.lr * g;
    }
  } else {
    v = h.alpha * v + (1.f - h.alpha) * g * g;
    w -= h.lr * g / (sqrtf(v) + h.eps);
  }
}

}  // namespace dlvk
