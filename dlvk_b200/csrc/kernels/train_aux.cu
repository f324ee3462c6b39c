// Training helpers that live on the device so a captured step graph can
// replay them: loss scaling by a device-resident scale, and fused L1/L2
// regularisation of the flat gradient buffer.
//
// Reference: GradientScaler::scale_loss (include/dlvk/training/
// mixed_precision.h:47-50) and L1/L2/ElasticNet regularizers
// (src/training/regularization.cpp:28-126: L1 loss lambda*sum|w| with
// gradient lambda*sign(w); L2 loss 0.5*lambda*sum w^2 with gradient
// lambda*w).  The reference downloads every weight to the host for these;
// here each is one pass over HBM.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

template <typename T>
__global__ void scale_dev_kernel(T* __restrict__ x, int64_t n, const float* __restrict__ s) {
  const float k = *s;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = from_f32<T>(to_f32(x[i]) * k);
}

template <typename TG>
__global__ void regularize_kernel(const float* __restrict__ w, TG* __restrict__ g, int64_t n, float l1, float l2,
                                  float ll1, float ll2, float* __restrict__ loss_out,
                                  const float* __restrict__ gscale) {
  __shared__ float sm[32];
  // Gradients that still carry a loss scale get the penalty's gradient at
  // that scale; the loss term itself is unscaled.
  const float k = gscale ? *gscale : 1.f;
  const float gl1 = l1 * k, gl2 = l2 * k;
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float x = w[i];
    const float sg = (x > 0.f) ? 1.f : ((x < 0.f) ? -1.f : 0.f);
    g[i] = from_f32<TG>(to_f32(g[i]) + gl1 * sg + gl2 * x);
    acc += ll1 * fabsf(x) + 0.5f * ll2 * x * x;
  }
  if (loss_out) {
    acc = block_sum(acc, sm);
    if (threadIdx.x == 0) atomicAdd(loss_out, acc);
  }
}

// One warp per row: argmax of the logits against the label (int id, or the
// argmax of a target-probability row).  Ties resolve to the lowest index.
template <typename T>
__global__ void step_metrics_kernel(const T* __restrict__ logits, int64_t rows, int cols, const int* __restrict__ labels,
                                    const float* __restrict__ probs, const float* __restrict__ loss,
                                    float* __restrict__ loss_sum, unsigned long long* __restrict__ correct,
                                    float loss_weight) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && loss && loss_sum) *loss_sum += *loss * loss_weight;
  if (!correct || (!labels && !probs)) return;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  unsigned int hits = 0;
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const T* row = logits + r * cols;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    float tbest = -INFINITY;
    int ti = 0x7fffffff;
    for (int c = lane; c < cols; c += 32) {
      const float v = to_f32(row[c]);
      if (v > best) { best = v; bi = c; }
      if (probs) {
        const float t = probs[r * cols + c];
        if (t > tbest) { tbest = t; ti = c; }
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      if (probs) {
        const float ot = __shfl_xor_sync(0xffffffffu, tbest, o);
        const int oti = __shfl_xor_sync(0xffffffffu, ti, o);
        if (ot > tbest || (ot == tbest && oti < ti)) { tbest = ot; ti = oti; }
      }
    }
    const int want = probs ? ti : labels[r];
    if (lane == 0 && bi == want) ++hits;
  }
  if (lane == 0 && hits) atomicAdd(correct, (unsigned long long)hits);
}

int grid_of(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8)); }

}  // namespace

void scale_by_device_scalar(DType dt, void* x, int64_t n, const float* s, cudaStream_t st) {
  if (n == 0) return;
  if (dt == DType::F32)
    scale_dev_kernel<float><<<grid_of(n), 256, 0, st>>>((float*)x, n, s);
  else if (dt == DType::BF16)
    scale_dev_kernel<__nv_bfloat16><<<grid_of(n), 256, 0, st>>>((__nv_bfloat16*)x, n, s);
  else
    throw std::runtime_error("dlvk::scale_by_device_scalar: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void regularize(const float* w, void* g, DType g_dt, int64_t n, float l1, float l2, float ll1, float ll2,
                float* loss_out, cudaStream_t s, const float* gscale) {
  if (n == 0) return;
  if (g_dt == DType::F32)
    regularize_kernel<float><<<grid_of(n), 256, 0, s>>>(w, (float*)g, n, l1, l2, ll1, ll2, loss_out, gscale);
  else if (g_dt == DType::BF16)
    regularize_kernel<__nv_bfloat16><<<grid_of(n), 256, 0, s>>>(w, (__nv_bfloat16*)g, n, l1, l2, ll1, ll2, loss_out,
                                                                 gscale);
  else
    throw std::runtime_error("dlvk::regularize: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void step_metrics(DType dt, const void* logits, int64_t rows, int cols, const int* labels, const float* probs,
                  const float* loss, float* loss_sum, unsigned long long* correct, float loss_weight, cudaStream_t s) {
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 148 * 4));
  if (dt == DType::F32)
    step_metrics_kernel<float><<<blocks, 256, 0, s>>>((const float*)logits, rows, cols, labels, probs, loss, loss_sum,
                                                      correct, loss_weight);
  else if (dt == DType::BF16)
    step_metrics_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)logits, rows, cols, labels, probs,
                                                              loss, loss_sum, correct, loss_weight);
  else
    throw std::runtime_error("dlvk::step_metrics: unsupported dtype");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
