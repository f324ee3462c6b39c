// Optimizer update kernels over flat parameter storage: Adam, SGD(-momentum),
// RMSprop; plus the gradient statistics used by clipping and loss scaling.
//
// Reference: shaders/adam_update.comp:31-61 (m, v, bias-corrected step; the
// host passes bc1 = bc2 = 1 at src/tensor/tensor_ops.cpp:2338-2357), SGD
// momentum in src/optimizers/sgd.cpp:55-76 (v = mu v + g; p -= lr v),
// RMSprop declared in include/dlvk/optimizers/optimizers.h:107-141,
// clipping in src/optimizers/optimizers.cpp:9-55.
//
// Hyper-parameters live in a small device struct (OptimHyper) so that one
// captured CUDA graph can replay many steps: `optim_advance` bumps the step
// counter and bias corrections on the device, the update kernels read them.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

__global__ void advance_kernel(OptimHyper* h) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    // A step that a loss scaler skips (non-finite gradients) does not count.
    if (h->skip_flag_ptr && *h->skip_flag_ptr) return;
    h->step += 1;
    const float t = (float)h->step;
    if (h->bias_correction) {
      h->bc1 = 1.f / (1.f - powf(h->beta1, t));
      h->bc2 = 1.f / (1.f - powf(h->beta2, t));
    } else {
      h->bc1 = 1.f;
      h->bc2 = 1.f;
    }
  }
}

template <typename TG>
__device__ __forceinline__ float load_grad(const TG* g, int64_t i) { return to_f32(g[i]); }

// Shared update rule used by the standalone kernels and by the fused
// all-reduce + optimizer kernel (comm.cu).
template <typename TG>
__global__ void update_kernel(int kind, const OptimHyper* __restrict__ h, float* __restrict__ p,
                              const TG* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                              __nv_bfloat16* __restrict__ p_bf16, int64_t n, float extra_scale) {
  const float lr = h->lr, b1 = h->beta1, b2 = h->beta2, eps = h->eps, wd = h->weight_decay;
  float gs = h->grad_scale * extra_scale;
  if (h->clip_coef_ptr) gs *= *h->clip_coef_ptr;
  if (h->skip_flag_ptr && *h->skip_flag_ptr) return;  // overflow detected: skip this step
  const float bc1 = h->bc1, bc2 = h->bc2, mom = h->momentum, alpha = h->alpha;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // Vector path: 4 elements per thread with 16-byte accesses (flat parameter
  // buffers and bucket boundaries are 256-byte aligned).
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                     reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15) == 0 &&
                   ((reinterpret_cast<uintptr_t>(p_bf16) & 7) == 0);
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n / 4;
    for (int64_t i4 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i4 < n4; i4 += stride) {
      float4 w = reinterpret_cast<const float4*>(p)[i4];
      float gg[4];
      if (sizeof(TG) == 4) {
        const float4 t = reinterpret_cast<const float4*>(g)[i4];
        gg[0] = t.x; gg[1] = t.y; gg[2] = t.z; gg[3] = t.w;
      } else {
        const uint2 t = reinterpret_cast<const uint2*>(g)[i4];
        const TG* e = reinterpret_cast<const TG*>(&t);
#pragma unroll
        for (int k = 0; k < 4; ++k) gg[k] = to_f32(e[k]);
      }
      float* wv = reinterpret_cast<float*>(&w);
      float4 mm4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = mm4;
      if (m) mm4 = reinterpret_cast<const float4*>(m)[i4];
      if (v) vv4 = reinterpret_cast<const float4*>(v)[i4];
      float* mv = reinterpret_cast<float*>(&mm4);
      float* vvv = reinterpret_cast<float*>(&vv4);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float gr = gg[k] * gs;
        if (wd != 0.f && !h->decoupled_wd) gr += wd * wv[k];
        if (kind == OPT_ADAM) {
          mv[k] = b1 * mv[k] + (1.f - b1) * gr;
          vvv[k] = b2 * vvv[k] + (1.f - b2) * gr * gr;
          if (wd != 0.f && h->decoupled_wd) wv[k] -= lr * wd * wv[k];
          wv[k] -= lr * (mv[k] * bc1) / (sqrtf(vvv[k] * bc2) + eps);
        } else if (kind == OPT_SGD) {
          if (mom != 0.f) {
            mv[k] = mom * mv[k] + gr;
            wv[k] -= lr * mv[k];
          } else {
            wv[k] -= lr * gr;
          }
        } else {
          vvv[k] = alpha * vvv[k] + (1.f - alpha) * gr * gr;
          wv[k] -= lr * gr / (sqrtf(vvv[k]) + eps);
        }
      }
      reinterpret_cast<float4*>(p)[i4] = w;
      if (m) reinterpret_cast<float4*>(m)[i4] = mm4;
      if (v) reinterpret_cast<float4*>(v)[i4] = vv4;
      if (p_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(wv[0], wv[1]), hi = __floats2bfloat162_rn(wv[2], wv[3]);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&lo);
        o.y = *reinterpret_cast<uint32_t*>(&hi);
        reinterpret_cast<uint2*>(p_bf16)[i4] = o;
      }
    }
    done = n4 * 4;
  }
  for (int64_t i = done + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float w = p[i];
    float gr = load_grad(g, i) * gs;
    if (wd != 0.f && !h->decoupled_wd) gr += wd * w;
    if (kind == OPT_ADAM) {
      const float mm = b1 * m[i] + (1.f - b1) * gr;
      const float vv = b2 * v[i] + (1.f - b2) * gr * gr;
      m[i] = mm;
      v[i] = vv;
      if (wd != 0.f && h->decoupled_wd) w -= lr * wd * w;
      w -= lr * (mm * bc1) / (sqrtf(vv * bc2) + eps);
    } else if (kind == OPT_SGD) {
      if (mom != 0.f) {
        const float vv = mom * m[i] + gr;
        m[i] = vv;
        w -= lr * vv;
      } else {
        w -= lr * gr;
      }
    } else {  // RMSprop
      const float sq = alpha * v[i] + (1.f - alpha) * gr * gr;
      v[i] = sq;
      w -= lr * gr / (sqrtf(sq) + eps);
    }
    p[i] = w;
    if (p_bf16) p_bf16[i] = __float2bfloat16_rn(w);
  }
}

// Per-block partial sum of squares and non-finite count of a gradient.
template <typename TG>
__global__ void grad_stats_partial(const TG* __restrict__ g, int64_t n, float* __restrict__ part_sq,
                                   int* __restrict__ part_bad) {
  __shared__ float sm[32];
  float acc = 0.f;
  int bad = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = to_f32(g[i]);
    if (!isfinite(x)) bad = 1;
    else acc += x * x;
  }
  acc = block_sum(acc, sm);
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    part_sq[blockIdx.x] = acc;
    part_bad[blockIdx.x] = bad;
  }
}

// Final: out[0] = total sum of squares * scale^2 (scale times *scale_ptr when
// given, e.g. a loss scaler's device-resident 1/scale), flag = any non-finite,
// clip = min(1, max_norm / (sqrt(sumsq) + 1e-6)) (if max_norm > 0).
__global__ void grad_stats_final(const float* __restrict__ part_sq, const int* __restrict__ part_bad, int nparts,
                                 float scale, const float* __restrict__ scale_ptr, float max_norm,
                                 float* __restrict__ sumsq_out, int* __restrict__ flag, float* __restrict__ clip_out,
                                 int accumulate) {
  __shared__ float sm[32];
  float acc = 0.f;
  int bad = 0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    acc += part_sq[i];
    bad |= part_bad[i];
  }
  acc = block_sum(acc, sm);
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    if (scale_ptr) scale *= *scale_ptr;
    float tot = acc * scale * scale;
    if (accumulate) tot += *sumsq_out;
    *sumsq_out = tot;
    if (flag) *flag = (accumulate ? *flag : 0) | bad;
    if (clip_out) {
      const float norm = sqrtf(tot);
      *clip_out = (max_norm > 0.f) ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    }
  }
}

// Dynamic loss scaling (GradientScaler semantics of
// include/dlvk/training/mixed_precision.h:15-60: init 65536, x2 every
// `interval` clean steps, x0.5 on overflow, clamped to [min, max]).
__global__ void scaler_update_kernel(float* scale, int* good_steps, const int* found_inf, float growth,
                                     float backoff, int interval, float smin, float smax, float* inv_scale) {
  if (threadIdx.x != 0) return;
  float s = *scale;
  if (*found_inf) {
    s = fmaxf(smin, s * backoff);
    *good_steps = 0;
  } else {
    int gsteps = *good_steps + 1;
    if (gsteps >= interval) {
      s = fminf(smax, s * growth);
      gsteps = 0;
    }
    *good_steps = gsteps;
  }
  *scale = s;
  if (inv_scale) *inv_scale = 1.f / s;
}

int update_grid(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, 148 * 16)); }

}  // namespace

void optim_advance(OptimHyper* h_dev, cudaStream_t s) {
  advance_kernel<<<1, 32, 0, s>>>(h_dev);
  DLVK_POST_LAUNCH();
}

void optim_update(int kind, const OptimHyper* h_dev, float* p, const void* g, DType g_dt, float* m, float* v,
                  __nv_bfloat16* p_bf16, int64_t n, float extra_scale, cudaStream_t s, int max_ctas) {
  if (n == 0) return;
  const int grid = max_ctas > 0 ? std::min(update_grid(n), max_ctas) : update_grid(n);
  if (g_dt == DType::F32)
    update_kernel<float><<<grid, 256, 0, s>>>(kind, h_dev, p, (const float*)g, m, v, p_bf16, n, extra_scale);
  else if (g_dt == DType::BF16)
    update_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(kind, h_dev, p, (const __nv_bfloat16*)g, m, v, p_bf16, n,
                                                      extra_scale);
  else
    throw std::runtime_error("dlvk::optim_update: unsupported grad dtype");
  DLVK_POST_LAUNCH();
}

int grad_stats_scratch_floats() { return 2 * 1024; }

void grad_stats(const void* g, DType g_dt, int64_t n, float scale, float max_norm, float* sumsq_out, int* flag,
                float* clip_out, bool accumulate, float* scratch, cudaStream_t s, const float* scale_ptr) {
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(1024, (n + 4095) / 4096));
  float* part_sq = scratch;
  int* part_bad = reinterpret_cast<int*>(scratch + 1024);
  if (g_dt == DType::F32)
    grad_stats_partial<float><<<blocks, 256, 0, s>>>((const float*)g, n, part_sq, part_bad);
  else if (g_dt == DType::BF16)
    grad_stats_partial<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)g, n, part_sq, part_bad);
  else
    throw std::runtime_error("dlvk::grad_stats: unsupported dtype");
  DLVK_POST_LAUNCH();
  grad_stats_final<<<1, 1024, 0, s>>>(part_sq, part_bad, blocks, scale, scale_ptr, max_norm, sumsq_out, flag, clip_out,
                                      accumulate ? 1 : 0);
  DLVK_POST_LAUNCH();
}

void scaler_update(float* scale, int* good_steps, const int* found_inf, float growth, float backoff, int interval,
                   float smin, float smax, float* inv_scale, cudaStream_t s) {
  scaler_update_kernel<<<1, 32, 0, s>>>(scale, good_steps, found_inf, growth, backoff, interval, smin, smax,
                                        inv_scale);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
