// Batch norm (fused with ReLU and Philox dropout), layer norm, standalone
// dropout and embedding kernels.
//
// Reference: shaders/batch_norm.comp:49-109 and batch_norm_backward.comp:49-136
// (feature-contiguous layout; layers use a CPU path, src/layers/
// batch_norm_layers.cpp:65-137 with an identity backward stub),
// shaders/layer_norm.comp:31-92 (backward stub, src/layers/modern_layers.cpp:
// 114-122), shaders/dropout.comp:38-66 (xorshift), dropout_backward.comp,
// shaders/embedding_lookup.comp:24-55 (backward returns nullptr,
// modern_layers.cpp:61-67).
//
// Dropout keep masks are never stored: element i of a call uses Philox4x32-10
// with key = seed and counter = {i/4 (64-bit), stream id, step}, lane i%4;
// keep iff u >= p.  The backward pass regenerates the same mask.  The step
// comes from device memory (`step_ptr`) so a captured CUDA graph draws fresh
// masks on every replay.
#include <cstdlib>

#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/sm100.h"

namespace dlvk {
namespace {

__device__ __forceinline__ uint4 philox_block(uint64_t blk, uint32_t stream, uint32_t step, uint64_t seed) {
  return philox4x32_10(make_uint4((uint32_t)blk, (uint32_t)(blk >> 32), stream, step),
                       make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
}
__device__ __forceinline__ uint32_t pick(const uint4& r, int j) {
  return j == 0 ? r.x : (j == 1 ? r.y : (j == 2 ? r.z : r.w));
}
__device__ __forceinline__ bool keep_elem(int64_t i, const DropoutDesc& d, uint32_t step) {
  const uint4 r = philox_block((uint64_t)i >> 2, d.stream, step, d.seed);
  return u01(pick(r, (int)(i & 3))) >= d.p;
}
__device__ __forceinline__ uint32_t read_step(const DropoutDesc& d) {
  return d.step_ptr ? (uint32_t)(*d.step_ptr) : d.step;
}

// ------------------------------------------------------------------ batch norm
// Scalar fallbacks of the element-wise passes (odd totals, unaligned
// tensors); same coefficients and masks as the 8-wide kernels.
template <typename T>
__global__ void bn_apply_kernel(const T* __restrict__ x, const float* __restrict__ scale,
                                const float* __restrict__ shift, T* __restrict__ y, int64_t total, int C, int S,
                                int relu, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / S) % C);
    float v = fmaf(to_f32(x[i]), scale[c], shift[c]);
    if (relu) v = fmaxf(v, 0.f);
    if (dd.p > 0.f) v = keep_elem(i, dd, step) ? v * inv_keep : 0.f;
    y[i] = from_f32<T>(v);
  }
}

template <typename T>
__global__ void bn_bwd_apply_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ A,
                                    const float* __restrict__ B, const float* __restrict__ D,
                                    const float* __restrict__ shift, T* __restrict__ dx, int64_t total, int C, int S,
                                    int relu, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / S) % C);
    const float xv = to_f32(x[i]);
    float g = to_f32(dy[i]);
    if (dd.p > 0.f) g = keep_elem(i, dd, step) ? g * inv_keep : 0.f;
    if (relu && !(fmaf(xv, A[c], shift[c]) > 0.f)) g = 0.f;
    dx[i] = from_f32<T>(fmaf(A[c], g, fmaf(B[c], xv, D[c])));
  }
}

// ---- BatchNorm, wide grids ---------------------------------------------------
// The reductions run in two passes: per-chunk partial sums over a 2-D grid
// (channel group x row chunk), then one thread per channel adds the chunks.
// The element-wise passes move 8 elements per thread (16-byte bf16 accesses)
// and draw the dropout mask one Philox block per 4 elements.

// Keep flags of elements i0 .. i0+7 (i0 a multiple of 4): the same mask as
// keep_elem() element by element.
__device__ __forceinline__ void keep8(int64_t i0, const DropoutDesc& d, uint32_t step, bool k[8]) {
  const uint4 r0 = philox_block((uint64_t)i0 >> 2, d.stream, step, d.seed);
  const uint4 r1 = philox_block(((uint64_t)i0 >> 2) + 1, d.stream, step, d.seed);
  k[0] = u01(r0.x) >= d.p; k[1] = u01(r0.y) >= d.p; k[2] = u01(r0.z) >= d.p; k[3] = u01(r0.w) >= d.p;
  k[4] = u01(r1.x) >= d.p; k[5] = u01(r1.y) >= d.p; k[6] = u01(r1.z) >= d.p; k[7] = u01(r1.w) >= d.p;
}
__device__ __forceinline__ void load8(const float* p, float v[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float v[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float* p, const float v[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float v[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

constexpr int BN_GROUP = 256;  // channels per block when S == 1 (8 per thread, 32 threads)

// Pass 1.  MODE 0 (statistics): a = sum(x - x0), b = sum((x - x0)^2) with x0
// the channel's first element (shifted sums keep the variance stable).
// MODE 1 (backward): a = sum(g), b = sum(g * xhat), g the upstream gradient
// through dropout and ReLU.  Grid (groups, chunks); `per` is rows per chunk
// when S == 1 (a group is BN_GROUP channels, 8 row lanes per block) and
// elements of the channel per chunk when S > 1 (a group is one channel).
// Output: part[chunk * C + c] (a) and part[(chunks + chunk) * C + c] (b).
template <typename T, int MODE>
__global__ void __launch_bounds__(256) bn_partial_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                                         const float* __restrict__ mean,
                                                         const float* __restrict__ rstd,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ beta, int N, int C, int S,
                                                         int64_t per, int relu, DropoutDesc dd, int vec,
                                                         float* __restrict__ part) {
  const uint32_t step = MODE == 1 ? read_step(dd) : 0u;
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  const int chunk = blockIdx.y, chunks = gridDim.y;
  if (S == 1) {
    __shared__ float sa[8][BN_GROUP + 1], sb[8][BN_GROUP + 1];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c0 = blockIdx.x * BN_GROUP + tx * 8;
    float a[8], b[8], k0[8], k1[8], k2[8], k3[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = min(c0 + j, C - 1);
      a[j] = b[j] = 0.f;
      if (MODE == 0) {
        k0[j] = to_f32(x[c]);
      } else {
        k0[j] = mean[c];
        k1[j] = rstd[c];
        k2[j] = (gamma ? gamma[c] : 1.f) * k1[j];      // the forward's scale
        k3[j] = (beta ? beta[c] : 0.f) - k0[j] * k2[j];  // and shift
      }
    }
    const int64_t n0 = (int64_t)chunk * per, n1 = min((int64_t)N, n0 + per);
    if (c0 < C) {
#pragma unroll 2
      for (int64_t n = n0 + ty; n < n1; n += 8) {
        const int64_t i0 = n * C + c0;
        float xv[8], gv[8];
        bool keep[8];
        if (vec) {
          load8(x + i0, xv);
          if (MODE == 1) {
            load8(dy + i0, gv);
            if (dd.p > 0.f) keep8(i0, dd, step, keep);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const bool in = c0 + j < C;
            xv[j] = in ? to_f32(x[i0 + j]) : 0.f;
            if (MODE == 1) {
              gv[j] = in ? to_f32(dy[i0 + j]) : 0.f;
              keep[j] = dd.p > 0.f && in ? keep_elem(i0 + j, dd, step) : true;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (c0 + j >= C) continue;
          if (MODE == 0) {
            const float v = xv[j] - k0[j];
            a[j] += v;
            b[j] += v * v;
          } else {
            const float xh = (xv[j] - k0[j]) * k1[j];
            float g = gv[j];
            if (dd.p > 0.f) g = keep[j] ? g * inv_keep : 0.f;
            if (relu && !(fmaf(xv[j], k2[j], k3[j]) > 0.f)) g = 0.f;
            a[j] += g;
            b[j] += g * xh;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sa[ty][tx * 8 + j] = a[j];
      sb[ty][tx * 8 + j] = b[j];
    }
    __syncthreads();
    const int cl = threadIdx.x, c = blockIdx.x * BN_GROUP + cl;
    if (c < C) {
      float ra = 0.f, rb = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        ra += sa[r][cl];
        rb += sb[r][cl];
      }
      part[(int64_t)chunk * C + c] = ra;
      part[(int64_t)(chunks + chunk) * C + c] = rb;
    }
  } else {
    __shared__ float sm[32];
    const int c = blockIdx.x;
    const int64_t cnt = (int64_t)N * S;
    const int64_t k0 = (int64_t)chunk * per, k1 = min(cnt, k0 + per);
    float sh = 0.f, mu = 0.f, rs = 0.f, sc = 1.f, sf = 0.f;
    if (MODE == 0) {
      sh = to_f32(x[(int64_t)c * S]);
    } else {
      mu = mean[c];
      rs = rstd[c];
      sc = (gamma ? gamma[c] : 1.f) * rs;
      sf = (beta ? beta[c] : 0.f) - mu * sc;
    }
    float a = 0.f, b = 0.f;
    for (int64_t k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
      const int64_t n = k / S, sp = k - n * S;
      const int64_t i = (n * C + c) * S + sp;
      if (MODE == 0) {
        const float v = to_f32(x[i]) - sh;
        a += v;
        b += v * v;
      } else {
        const float xv = to_f32(x[i]);
        const float xh = (xv - mu) * rs;
        float g = to_f32(dy[i]);
        if (dd.p > 0.f) g = keep_elem(i, dd, step) ? g * inv_keep : 0.f;
        if (relu && !(fmaf(xv, sc, sf) > 0.f)) g = 0.f;
        a += g;
        b += g * xh;
      }
    }
    a = block_sum(a, sm);
    b = block_sum(b, sm);
    if (threadIdx.x == 0) {
      part[(int64_t)chunk * C + c] = a;
      part[(int64_t)(chunks + chunk) * C + c] = b;
    }
  }
}

// Per-channel coefficients of the element-wise passes, so that every element
// costs one fma per term:
//   forward   pre = fma(x, scale, shift), scale = gamma * rstd,
//             shift = beta - mean * scale;  y = dropout(relu(pre))
//   backward  dx = A * g + B * x + D with g the masked upstream gradient,
//             A = gamma * rstd, B = -A * rstd * sgx / M,
//             D = -A * sg / M - B * mean  (the ReLU test reuses pre).
// Scratch layout (floats): [scale | shift | A | B | D | sg | sgx | partials].
struct BnCoef {
  float* scale;
  float* shift;
  float* A;
  float* B;
  float* D;
  float* sg;
  float* sgx;
  float* part;
};
__host__ __device__ inline BnCoef bn_coef(float* scratch, int C) {
  return BnCoef{scratch, scratch + C, scratch + 2 * (int64_t)C, scratch + 3 * (int64_t)C, scratch + 4 * (int64_t)C,
                scratch + 5 * (int64_t)C, scratch + 6 * (int64_t)C, scratch + 7 * (int64_t)C};
}

// Sum of the chunk partials of 32 channels per block, 8 lanes per channel.
__device__ __forceinline__ bool bn_sum_chunks(const float* __restrict__ part, int chunks, int C, float& a, float& b) {
  __shared__ float sa[8][33], sb[8][33];
  const int cl = threadIdx.x & 31, ly = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  a = 0.f;
  b = 0.f;
  if (c < C)
    for (int k = ly; k < chunks; k += 8) {
      a += part[(int64_t)k * C + c];
      b += part[(int64_t)(chunks + k) * C + c];
    }
  sa[ly][cl] = a;
  sb[ly][cl] = b;
  __syncthreads();
  if (ly != 0 || c >= C) return false;
#pragma unroll
  for (int r = 1; r < 8; ++r) {
    a += sa[r][cl];
    b += sb[r][cl];
  }
  return true;
}

// Pass 2 of the statistics: mean, rstd, the running averages and the forward
// coefficients.  The running variance tracks the population (divide-by-count)
// variance, as the reference's layer does (src/layers/batch_norm_layers.cpp:
// 79-90).
template <typename T>
__global__ void __launch_bounds__(256) bn_stats_finalize_kernel(const float* __restrict__ part, int chunks,
                                                                const T* __restrict__ x, int C, int S, int64_t count,
                                                                float* __restrict__ mean, float* __restrict__ rstd,
                                                                float* __restrict__ run_mean,
                                                                float* __restrict__ run_var, float momentum, float eps,
                                                                const float* __restrict__ gamma,
                                                                const float* __restrict__ beta, BnCoef co) {
  float a, b;
  if (!bn_sum_chunks(part, chunks, C, a, b)) return;
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  const float m1 = a / (float)count;
  const float var = fmaxf(b / (float)count - m1 * m1, 0.f);
  const float mu = m1 + to_f32(x[(int64_t)c * S]);
  const float rs = rsqrtf(var + eps);
  mean[c] = mu;
  rstd[c] = rs;
  if (run_mean) run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
  if (run_var) run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
  const float sc = (gamma ? gamma[c] : 1.f) * rs;
  co.scale[c] = sc;
  co.shift[c] = (beta ? beta[c] : 0.f) - mu * sc;
}

// Forward coefficients from given statistics (inference: running stats).
__global__ void bn_coef_kernel(const float* __restrict__ mean, const float* __restrict__ rstd,
                               const float* __restrict__ gamma, const float* __restrict__ beta, int C, BnCoef co) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const float sc = (gamma ? gamma[c] : 1.f) * rstd[c];
  co.scale[c] = sc;
  co.shift[c] = (beta ? beta[c] : 0.f) - mean[c] * sc;
}

// Pass 2 of the backward reduction: sg, sgx, the parameter gradients and the
// backward coefficients.
__global__ void __launch_bounds__(256) bn_bwd_finalize_kernel(const float* __restrict__ part, int chunks, int C,
                                                              const float* __restrict__ mean,
                                                              const float* __restrict__ rstd,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float inv_count,
                                                              float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                              int accumulate, BnCoef co) {
  float a, b;
  if (!bn_sum_chunks(part, chunks, C, a, b)) return;
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  co.sg[c] = a;
  co.sgx[c] = b;
  if (dbeta) dbeta[c] = accumulate ? dbeta[c] + a : a;
  if (dgamma) dgamma[c] = accumulate ? dgamma[c] + b : b;
  const float rs = rstd[c], A = (gamma ? gamma[c] : 1.f) * rs;
  const float B = -A * rs * b * inv_count;
  co.A[c] = A;
  co.B[c] = B;
  co.D[c] = -A * a * inv_count - B * mean[c];
  co.shift[c] = (beta ? beta[c] : 0.f) - mean[c] * A;
}

// Channel of element i0 and its position inside the channel's S run.
__device__ __forceinline__ void bn_chan(int64_t i0, int C, int S, int& c, int& sp) {
  if (S == 1) {
    c = (int)(i0 % C);
    sp = 0;
  } else {
    const int64_t q = i0 / S;
    sp = (int)(i0 - q * S);
    c = (int)(q % C);
  }
}
__device__ __forceinline__ void bn_next(int C, int S, int& c, int& sp) {
  if (++sp >= S) {
    sp = 0;
    if (++c == C) c = 0;
  }
}
// Coefficients of the 8 elements from i0: one pair of float4 loads per array
// when the 8 elements are 8 consecutive channels (S == 1, C % 8 == 0).
template <int NA>
__device__ __forceinline__ void bn_coef8(const float* const (&arr)[NA], int64_t i0, int C, int S, bool chan8,
                                         float (&o)[NA][8]) {
  if (chan8) {
    const int c0 = (int)(i0 % C);
#pragma unroll
    for (int a = 0; a < NA; ++a) load8(arr[a] + c0, o[a]);
  } else {
    int c, sp;
    bn_chan(i0, C, S, c, sp);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int a = 0; a < NA; ++a) o[a][j] = arr[a][c];
      bn_next(C, S, c, sp);
    }
  }
}

// y = dropout(relu(x * scale + shift)), 8 elements per thread (total % 8 == 0,
// 16-byte aligned x and y).
template <typename T>
__global__ void bn_apply_vec_kernel(const T* __restrict__ x, BnCoef co, T* __restrict__ y, int64_t total, int C,
                                    int S, int relu, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  const bool chan8 = S == 1 && (C & 7) == 0;
  const float* const arr[2] = {co.scale, co.shift};
  const int64_t n8 = total >> 3;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n8; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = t << 3;
    float v[8], k[2][8];
    bool keep[8];
    load8(x + i0, v);
    bn_coef8<2>(arr, i0, C, S, chan8, k);
    if (dd.p > 0.f) keep8(i0, dd, step, keep);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float o = fmaf(v[j], k[0][j], k[1][j]);
      if (relu) o = fmaxf(o, 0.f);
      if (dd.p > 0.f) o = keep[j] ? o * inv_keep : 0.f;
      v[j] = o;
    }
    store8(y + i0, v);
  }
}

// dx = A * g + B * x + D, 8 elements per thread.
template <typename T>
__global__ void bn_bwd_apply_vec_kernel(const T* __restrict__ x, const T* __restrict__ dy, BnCoef co,
                                        T* __restrict__ dx, int64_t total, int C, int S, int relu, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  const bool chan8 = S == 1 && (C & 7) == 0;
  const float* const arr[4] = {co.A, co.B, co.D, co.shift};
  const int64_t n8 = total >> 3;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n8; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i0 = t << 3;
    float xv[8], gv[8], k[4][8];
    bool keep[8];
    load8(x + i0, xv);
    load8(dy + i0, gv);
    bn_coef8<4>(arr, i0, C, S, chan8, k);
    if (dd.p > 0.f) keep8(i0, dd, step, keep);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float g = gv[j];
      if (dd.p > 0.f) g = keep[j] ? g * inv_keep : 0.f;
      if (relu && !(fmaf(xv[j], k[0][j], k[3][j]) > 0.f)) g = 0.f;
      xv[j] = fmaf(k[0][j], g, fmaf(k[1][j], xv[j], k[2][j]));
    }
    store8(dx + i0, xv);
  }
}

// ------------------------------------------------------------------ layer norm
// One warp per row.
template <typename T>
__global__ void ln_fwd_kernel(const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
                              T* __restrict__ y, float* __restrict__ mean, float* __restrict__ rstd, int64_t rows,
                              int D, float eps) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const T* xr = x + r * D;
  const float shift = to_f32(xr[0]);
  float a = 0.f, b = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float v = to_f32(xr[d]) - shift;
    a += v;
    b += v * v;
  }
  a = warp_sum(a);
  b = warp_sum(b);
  const float m1 = a / D;
  const float mu = m1 + shift;
  const float rs = rsqrtf(fmaxf(b / D - m1 * m1, 0.f) + eps);
  T* yr = y + r * D;
  for (int d = lane; d < D; d += 32)
    yr[d] = from_f32<T>((to_f32(xr[d]) - mu) * rs * (gamma ? gamma[d] : 1.f) + (beta ? beta[d] : 0.f));
  if (lane == 0) {
    if (mean) mean[r] = mu;
    if (rstd) rstd[r] = rs;
  }
}

// Register-resident variant: one warp per row, D = 32 lanes x NV vectors of
// 16 bytes; exact two-pass mean / variance from registers, 16-byte loads and
// stores, gamma / beta as float4.
template <typename T, int NV>
__global__ void __launch_bounds__(256, 4) ln_fwd_vec_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, T* __restrict__ y,
                                                            float* __restrict__ mean, float* __restrict__ rstd,
                                                            int64_t rows, int D, float eps) {
  // One warp per row; the row stays in registers as raw 16-byte vectors and
  // is converted on each of the three passes (mean, variance, output), which
  // keeps registers low enough for four blocks (32 warps) per SM.
  pdl_wait();
  constexpr int EPV = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    uint4 u[NV];
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * D);
#pragma unroll
    for (int k = 0; k < NV; ++k) u[k] = xr[k * 32 + lane];
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const T* e = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
      for (int j = 0; j < EPV; ++j) a += to_f32(e[j]);
    }
    const float mu = warp_sum(a) / D;
    float b = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const T* e = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
      for (int j = 0; j < EPV; ++j) {
        const float d0 = to_f32(e[j]) - mu;
        b += d0 * d0;
      }
    }
    const float rs = rsqrtf(warp_sum(b) / D + eps);
    uint4* yr = reinterpret_cast<uint4*>(y + r * D);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int d0 = (k * 32 + lane) * EPV;
      const T* e = reinterpret_cast<const T*>(&u[k]);
      uint4 o;
      T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < EPV; j += 4) {
        const float4 g4 = gamma ? *reinterpret_cast<const float4*>(gamma + d0 + j) : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 b4 = beta ? *reinterpret_cast<const float4*>(beta + d0 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        eo[j] = from_f32<T>((to_f32(e[j]) - mu) * rs * g4.x + b4.x);
        eo[j + 1] = from_f32<T>((to_f32(e[j + 1]) - mu) * rs * g4.y + b4.y);
        eo[j + 2] = from_f32<T>((to_f32(e[j + 2]) - mu) * rs * g4.z + b4.z);
        eo[j + 3] = from_f32<T>((to_f32(e[j + 3]) - mu) * rs * g4.w + b4.w);
      }
      yr[k * 32 + lane] = o;
    }
    if (lane == 0) {
      if (mean) mean[r] = mu;
      if (rstd) rstd[r] = rs;
    }
  }
}

// Rows of up to 1024 bf16 / 512 fp32 elements: gamma / beta staged in shared
// memory once per block, and every warp loads all R of its rows before
// reducing any, so a [rows <= grid warps * R] tensor costs one DRAM round trip
// per warp (13.3 us against 14.4 us for one row at a time at [8192 x 1024]
// bf16, L2 cold; a plain 16 MB -> 16 MB copy takes 10.3 us).
template <typename T, int NV, int R>
__global__ void __launch_bounds__(256, 2) ln_fwd_rows_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                             const float* __restrict__ beta, T* __restrict__ y,
                                                             float* __restrict__ mean, float* __restrict__ rstd,
                                                             int64_t rows, int D, float eps) {
  extern __shared__ float4 sgb[];  // gamma as D / 4 float4, then beta
  constexpr int EPV = 16 / sizeof(T);
  const int n4 = D / 4;
  pdl_wait();
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    sgb[i] = gamma ? reinterpret_cast<const float4*>(gamma)[i] : make_float4(1.f, 1.f, 1.f, 1.f);
    sgb[n4 + i] = beta ? reinterpret_cast<const float4*>(beta)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r0 < rows; r0 += warps * R) {
    uint4 u[R][NV];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int64_t r = r0 + j * warps;
      const uint4* xr = reinterpret_cast<const uint4*>(x + r * D);
#pragma unroll
      for (int k = 0; k < NV; ++k) u[j][k] = r < rows ? xr[k * 32 + lane] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int64_t r = r0 + j * warps;
      if (r >= rows) break;  // warp-uniform
      float a = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const T* e = reinterpret_cast<const T*>(&u[j][k]);
#pragma unroll
        for (int t = 0; t < EPV; ++t) a += to_f32(e[t]);
      }
      const float mu = warp_sum(a) / D;
      float b = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const T* e = reinterpret_cast<const T*>(&u[j][k]);
#pragma unroll
        for (int t = 0; t < EPV; ++t) {
          const float d0 = to_f32(e[t]) - mu;
          b += d0 * d0;
        }
      }
      const float rs = rsqrtf(warp_sum(b) / D + eps);
      uint4* yr = reinterpret_cast<uint4*>(y + r * D);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int q0 = (k * 32 + lane) * (EPV / 4);  // first float4 of gamma / beta for this vector
        const T* e = reinterpret_cast<const T*>(&u[j][k]);
        uint4 o;
        T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int t = 0; t < EPV; t += 4) {
          const float4 g4 = sgb[q0 + t / 4], b4 = sgb[n4 + q0 + t / 4];
          eo[t] = from_f32<T>((to_f32(e[t]) - mu) * rs * g4.x + b4.x);
          eo[t + 1] = from_f32<T>((to_f32(e[t + 1]) - mu) * rs * g4.y + b4.y);
          eo[t + 2] = from_f32<T>((to_f32(e[t + 2]) - mu) * rs * g4.z + b4.z);
          eo[t + 3] = from_f32<T>((to_f32(e[t + 3]) - mu) * rs * g4.w + b4.w);
        }
        yr[k * 32 + lane] = o;
      }
      if (lane == 0) {
        if (mean) mean[r] = mu;
        if (rstd) rstd[r] = rs;
      }
    }
  }
}

// dx per row (one warp per row, grid-stride over rows with a fixed grid);
// each block accumulates dgamma/dbeta partials for its rows in shared memory
// and writes them to part[block][2*D].  Fixed order => deterministic.
template <typename T>
__global__ void ln_bwd_kernel(const T* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ mean,
                              const float* __restrict__ rstd, const T* __restrict__ dy, T* __restrict__ dx,
                              float* __restrict__ part, int64_t rows, int D, const T* __restrict__ dres) {
  extern __shared__ float sp[];  // [warps][2*D]
  const int warps = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* mine = sp + (int64_t)w * 2 * D;
  for (int d = lane; d < 2 * D; d += 32) mine[d] = 0.f;
  for (int64_t r = (int64_t)blockIdx.x * warps + w; r < rows; r += (int64_t)gridDim.x * warps) {
    const T* xr = x + r * D;
    const T* gr = dy + r * D;
    const float mu = mean[r], rs = rstd[r];
    float a = 0.f, b = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float xh = (to_f32(xr[d]) - mu) * rs;
      const float g = to_f32(gr[d]);
      const float gg = g * (gamma ? gamma[d] : 1.f);
      a += gg;
      b += gg * xh;
      mine[d] += g * xh;
      mine[D + d] += g;
    }
    a = warp_sum(a) / D;
    b = warp_sum(b) / D;
    T* dr = dx + r * D;
    for (int d = lane; d < D; d += 32) {
      const float xh = (to_f32(xr[d]) - mu) * rs;
      const float gg = to_f32(gr[d]) * (gamma ? gamma[d] : 1.f);
      dr[d] = from_f32<T>(rs * (gg - a - xh * b) + (dres ? to_f32(dres[r * D + d]) : 0.f));
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < 2 * D; d += blockDim.x) {
    float s = 0.f;
    for (int i = 0; i < warps; ++i) s += sp[(int64_t)i * 2 * D + d];
    part[(int64_t)blockIdx.x * 2 * D + d] = s;
  }
}

// Register-resident variant for D = 32 * NV * EPV: lane l owns the 16-byte
// vectors l, l+32, ... of every row, so dgamma/dbeta partials stay in
// registers across the rows of a warp; the 8 warps of a block then combine
// them through shared memory in warp order and write one partial per block.
template <typename T, int NV>
__global__ void __launch_bounds__(256) ln_bwd_warp_kernel(const T* __restrict__ x, const float* __restrict__ gamma,
                                                          const float* __restrict__ mean,
                                                          const float* __restrict__ rstd, const T* __restrict__ dy,
                                                          T* __restrict__ dx, float* __restrict__ part, int64_t rows,
                                                          int D, const T* __restrict__ dres) {
  // One warp per row, the row held in registers; the next row's x, dy (and
  // residual gradient) are loaded before the current row is processed, so
  // two rows per warp are in flight.
  constexpr int EPV = 16 / sizeof(T);
  extern __shared__ float sp[];  // [8][2*D] partials, then gamma [D]
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sgam = sp + 16 * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) sgam[d] = gamma ? gamma[d] : 1.f;
  __syncthreads();
  float adg[NV][EPV], adb[NV][EPV];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      adg[i][k] = 0.f;
      adb[i][k] = 0.f;
    }
  const float invD = 1.f / D;
  const int64_t step = (int64_t)gridDim.x * 8;
  int64_t r = (int64_t)blockIdx.x * 8 + w;
  uint4 nx[NV], ng[NV], nr[NV];
  auto fetch = [&](int64_t row) {
    if (row >= rows) return;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      nx[i] = reinterpret_cast<const uint4*>(x + row * D)[lane + 32 * i];
      ng[i] = reinterpret_cast<const uint4*>(dy + row * D)[lane + 32 * i];
      if (dres) nr[i] = reinterpret_cast<const uint4*>(dres + row * D)[lane + 32 * i];
    }
  };
  fetch(r);
  for (; r < rows; r += step) {
    uint4 cx[NV], cg[NV], cr[NV];  // current row, raw; nx/ng/nr take the next one
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      cx[i] = nx[i];
      cg[i] = ng[i];
      cr[i] = nr[i];
    }
    const float mu = mean[r], rs = rstd[r];
    fetch(r + step);
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const T* ex = reinterpret_cast<const T*>(&cx[i]);
      const T* eg = reinterpret_cast<const T*>(&cg[i]);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (to_f32(ex[k]) - mu) * rs;
        const float g = to_f32(eg[k]);
        const float gg = g * sgam[(lane + 32 * i) * EPV + k];
        a += gg;
        b += gg * xh;
        adg[i][k] += g * xh;
        adb[i][k] += g;
      }
    }
    a = warp_sum(a) * invD;
    b = warp_sum(b) * invD;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const T* ex = reinterpret_cast<const T*>(&cx[i]);
      const T* eg = reinterpret_cast<const T*>(&cg[i]);
      const T* er = reinterpret_cast<const T*>(&cr[i]);
      uint4 o;
      T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (to_f32(ex[k]) - mu) * rs;
        const float v = rs * (to_f32(eg[k]) * sgam[(lane + 32 * i) * EPV + k] - a - xh * b);
        eo[k] = from_f32<T>(dres ? v + to_f32(er[k]) : v);
      }
      reinterpret_cast<uint4*>(dx + r * D)[lane + 32 * i] = o;
    }
  }
  float* mine = sp + (int64_t)w * 2 * D;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      const int col = (lane + 32 * i) * EPV + k;
      mine[col] = adg[i][k];
      mine[D + col] = adb[i][k];
    }
  __syncthreads();
  for (int d = threadIdx.x; d < 2 * D; d += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += sp[(int64_t)i * 2 * D + d];
    part[(int64_t)blockIdx.x * 2 * D + d] = s;
  }
}

// Deep-pipelined variant for bf16 rows of 256 x NV elements (D = 1024 with
// NV = 4): each warp streams its rows through a 3-slot shared-memory ring
// with cp.async (x, dy and the residual gradient of three rows in flight per
// warp, 8 warps and one CTA per SM), reading the row back from shared memory
// in both passes, so registers hold only the dgamma / dbeta accumulators.
// Every lane reads back only the 16-byte vectors it copied itself, so
// cp.async.wait_group alone orders the copy before the read.
template <int NV, bool RES>
__global__ void __launch_bounds__(256, 1) ln_bwd_ring_kernel(const __nv_bfloat16* __restrict__ x,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ mean,
                                                             const float* __restrict__ rstd,
                                                             const __nv_bfloat16* __restrict__ dy,
                                                             __nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                             int64_t rows, int D,
                                                             const __nv_bfloat16* __restrict__ dres) {
  // part: [blocks][PD] partials, dgamma | dbeta (| column sums of dres)
  constexpr int EPV = 8, RING = 3, NT = RES ? 3 : 2, RV = NV * 32;  // 16-byte vectors per tensor row
  constexpr int NP = RES ? 3 : 2;
  pdl_wait();
  extern __shared__ uint4 sring[];                                   // [8][RING][NT][RV]
  float* sgam = reinterpret_cast<float*>(sring + 8 * RING * NT * RV);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int d = threadIdx.x; d < D; d += blockDim.x) sgam[d] = gamma ? gamma[d] : 1.f;
  __syncthreads();
  uint4* ring = sring + (size_t)w * RING * NT * RV;
  const int64_t step = (int64_t)gridDim.x * 8;
  const int64_t r0 = (int64_t)blockIdx.x * 8 + w;
  auto issue = [&](int64_t row, int slot) {
    if (row < rows) {
      uint4* b = ring + slot * NT * RV;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int v = lane + 32 * i;
        sm100::cp_async_16(sm100::smem_u32(b + v), reinterpret_cast<const uint4*>(x + row * D) + v, 16);
        sm100::cp_async_16(sm100::smem_u32(b + RV + v), reinterpret_cast<const uint4*>(dy + row * D) + v, 16);
        if (RES)
          sm100::cp_async_16(sm100::smem_u32(b + 2 * RV + v), reinterpret_cast<const uint4*>(dres + row * D) + v, 16);
      }
    }
    sm100::cp_async_commit();  // empty groups keep the count aligned
  };
#pragma unroll
  for (int k = 0; k < RING; ++k) issue(r0 + k * step, k);
  // gr: this lane's gamma in registers (shared-memory reads at an 8-float
  // lane stride would conflict 8 ways on every element).
  // adr: column sums of dres (the bias gradient of the layer whose output
  // gradient dres is, when the block's residual sum ends in a biased GEMM).
  float adg[NV][EPV], adb[NV][EPV], adr[NV][EPV], gr[NV][EPV];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      adg[i][k] = adb[i][k] = adr[i][k] = 0.f;
      gr[i][k] = sgam[(lane + 32 * i) * EPV + k];
    }
  const float invD = 1.f / D;
  int slot = 0;
  for (int64_t r = r0; r < rows; r += step) {
    sm100::cp_async_wait<RING - 1>();
    const uint4* b = ring + slot * NT * RV;
    const float mu = mean[r], rs = rstd[r];
    float a = 0.f, bb = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint4 ux = b[lane + 32 * i], ug = b[RV + lane + 32 * i];
      const __nv_bfloat16* ex = reinterpret_cast<const __nv_bfloat16*>(&ux);
      const __nv_bfloat16* eg = reinterpret_cast<const __nv_bfloat16*>(&ug);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (__bfloat162float(ex[k]) - mu) * rs;
        const float g = __bfloat162float(eg[k]);
        const float gg = g * gr[i][k];
        a += gg;
        bb += gg * xh;
        adg[i][k] += g * xh;
        adb[i][k] += g;
      }
    }
    a = warp_sum(a) * invD;
    bb = warp_sum(bb) * invD;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint4 ux = b[lane + 32 * i], ug = b[RV + lane + 32 * i];
      uint4 ur = make_uint4(0, 0, 0, 0);
      if (RES) ur = b[2 * RV + lane + 32 * i];
      const __nv_bfloat16* ex = reinterpret_cast<const __nv_bfloat16*>(&ux);
      const __nv_bfloat16* eg = reinterpret_cast<const __nv_bfloat16*>(&ug);
      const __nv_bfloat16* er = reinterpret_cast<const __nv_bfloat16*>(&ur);
      uint4 o;
      __nv_bfloat16* eo = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (__bfloat162float(ex[k]) - mu) * rs;
        float v = rs * (__bfloat162float(eg[k]) * gr[i][k] - a - xh * bb);
        if (RES) {
          const float rv = __bfloat162float(er[k]);
          v += rv;
          adr[i][k] += rv;
        }
        eo[k] = __float2bfloat16_rn(v);
      }
      reinterpret_cast<uint4*>(dx + r * D)[lane + 32 * i] = o;
    }
    issue(r + RING * step, slot);  // this lane has read its vectors of the slot
    slot = slot + 1 == RING ? 0 : slot + 1;
  }
  sm100::cp_async_wait<0>();
  __syncthreads();
  float* sp = reinterpret_cast<float*>(sring);  // the ring is free: [8][NP*D] partials
  float* mine = sp + (int64_t)w * NP * D;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      const int col = (lane + 32 * i) * EPV + k;
      mine[col] = adg[i][k];
      mine[D + col] = adb[i][k];
      if (RES) mine[2 * D + col] = adr[i][k];
    }
  __syncthreads();
  for (int d = threadIdx.x; d < NP * D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += sp[(int64_t)i * NP * D + d];
    part[(int64_t)blockIdx.x * NP * D + d] = acc;
  }
}

// Two warps per row for bf16 rows of 512 x NVH elements (D = 512 or 1024;
// NVH = 1 or 2): warp 2p + h of a block owns columns [h D/2, (h+1) D/2) of the
// rows of pair p, so a lane holds 16 dgamma / dbeta (/ dres column-sum)
// accumulators instead of 32 and a block runs 16 warps.  Each warp streams
// its half rows (x, dy and the residual gradient, with the row's mean and
// rstd) through a 3-slot cp.async ring; the two halves of a row exchange
// their partial sums through shared memory under a named barrier of the
// pair's 64 threads (slot by row parity, so a write never races the
// partner's read of the previous row).  Partials per block as in
// ln_bwd_ring_kernel, so ln_bwd_final_kernel finishes both.
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
template <int NVH, bool RES>
__global__ void __launch_bounds__(512, 1) ln_bwd_pair_kernel(const __nv_bfloat16* __restrict__ x,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ mean,
                                                             const float* __restrict__ rstd,
                                                             const __nv_bfloat16* __restrict__ dy,
                                                             __nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                             int64_t rows, int D,
                                                             const __nv_bfloat16* __restrict__ dres) {
  constexpr int EPV = 8, RING = 3, NT = RES ? 3 : 2, RV = NVH * 32;  // 16-byte vectors per tensor half row
  constexpr int NP = RES ? 3 : 2;
  constexpr int HALF = RV * EPV;  // columns per half row
  pdl_wait();
  extern __shared__ uint4 sring[];                                   // [16][RING][NT][RV]
  float* sgam = reinterpret_cast<float*>(sring + 16 * RING * NT * RV);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pr = w >> 1, hh = w & 1;
  float* mystat = sgam + D + w * RING * 2;                            // [RING][mean, rstd]
  float2* xch = reinterpret_cast<float2*>(sgam + D + 16 * RING * 2);  // [8 pairs][2 parities][2 halves]
  for (int d = threadIdx.x; d < D; d += blockDim.x) sgam[d] = gamma ? gamma[d] : 1.f;
  __syncthreads();
  uint4* ring = sring + (size_t)w * RING * NT * RV;
  const int64_t step = (int64_t)gridDim.x * 8;
  const int64_t r0 = (int64_t)blockIdx.x * 8 + pr;
  const int col0 = hh * HALF;
  auto issue = [&](int64_t row, int slot) {
    if (row < rows) {
      uint4* b = ring + slot * NT * RV;
      const int64_t base = row * D + col0;
#pragma unroll
      for (int i = 0; i < NVH; ++i) {
        const int v = lane + 32 * i;
        sm100::cp_async_16(sm100::smem_u32(b + v), reinterpret_cast<const uint4*>(x + base) + v, 16);
        sm100::cp_async_16(sm100::smem_u32(b + RV + v), reinterpret_cast<const uint4*>(dy + base) + v, 16);
        if (RES)
          sm100::cp_async_16(sm100::smem_u32(b + 2 * RV + v), reinterpret_cast<const uint4*>(dres + base) + v, 16);
      }
      if (lane < 2)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sm100::smem_u32(mystat + slot * 2 + lane)),
                     "l"((lane ? rstd : mean) + row)
                     : "memory");
    }
    sm100::cp_async_commit();  // empty groups keep the count aligned
  };
#pragma unroll
  for (int k = 0; k < RING; ++k) issue(r0 + k * step, k);
  float adg[NVH][EPV], adb[NVH][EPV], adr[NVH][EPV], gr[NVH][EPV];
#pragma unroll
  for (int i = 0; i < NVH; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      adg[i][k] = adb[i][k] = adr[i][k] = 0.f;
      gr[i][k] = sgam[col0 + (lane + 32 * i) * EPV + k];
    }
  const float invD = 1.f / D;
  int slot = 0, par = 0;
  for (int64_t r = r0; r < rows; r += step, par ^= 1) {
    sm100::cp_async_wait<RING - 1>();
    __syncwarp();  // lanes 0 and 1 copied the row's mean and rstd
    const uint4* b = ring + slot * NT * RV;
    const float mu = mystat[slot * 2], rs = mystat[slot * 2 + 1];
    float a = 0.f, bb = 0.f;
#pragma unroll
    for (int i = 0; i < NVH; ++i) {
      const uint4 ux = b[lane + 32 * i], ug = b[RV + lane + 32 * i];
      const __nv_bfloat16* ex = reinterpret_cast<const __nv_bfloat16*>(&ux);
      const __nv_bfloat16* eg = reinterpret_cast<const __nv_bfloat16*>(&ug);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (__bfloat162float(ex[k]) - mu) * rs;
        const float g = __bfloat162float(eg[k]);
        const float gg = g * gr[i][k];
        a += gg;
        bb += gg * xh;
        adg[i][k] += g * xh;
        adb[i][k] += g;
      }
    }
    a = warp_sum(a);
    bb = warp_sum(bb);
    if (lane == 0) xch[(pr * 2 + par) * 2 + hh] = make_float2(a, bb);
    named_sync(1 + pr, 64);
    const float2 o = xch[(pr * 2 + par) * 2 + (hh ^ 1)];
    a = (a + o.x) * invD;
    bb = (bb + o.y) * invD;
#pragma unroll
    for (int i = 0; i < NVH; ++i) {
      const uint4 ux = b[lane + 32 * i], ug = b[RV + lane + 32 * i];
      uint4 ur = make_uint4(0, 0, 0, 0);
      if (RES) ur = b[2 * RV + lane + 32 * i];
      const __nv_bfloat16* ex = reinterpret_cast<const __nv_bfloat16*>(&ux);
      const __nv_bfloat16* eg = reinterpret_cast<const __nv_bfloat16*>(&ug);
      const __nv_bfloat16* er = reinterpret_cast<const __nv_bfloat16*>(&ur);
      uint4 ov;
      __nv_bfloat16* eo = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const float xh = (__bfloat162float(ex[k]) - mu) * rs;
        float v = rs * (__bfloat162float(eg[k]) * gr[i][k] - a - xh * bb);
        if (RES) {
          const float rv = __bfloat162float(er[k]);
          v += rv;
          adr[i][k] += rv;
        }
        eo[k] = __float2bfloat16_rn(v);
      }
      reinterpret_cast<uint4*>(dx + r * D + col0)[lane + 32 * i] = ov;
    }
    issue(r + RING * step, slot);  // this lane has read its vectors of the slot
    slot = slot + 1 == RING ? 0 : slot + 1;
  }
  sm100::cp_async_wait<0>();
  __syncthreads();
  float* sp = reinterpret_cast<float*>(sring);  // the ring is free: [16 warps][NP][HALF] partials
  float* mine = sp + (int64_t)w * NP * HALF;
#pragma unroll
  for (int i = 0; i < NVH; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      const int col = (lane + 32 * i) * EPV + k;
      mine[col] = adg[i][k];
      mine[HALF + col] = adb[i][k];
      if (RES) mine[2 * HALF + col] = adr[i][k];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < NP * D; idx += blockDim.x) {
    const int np = idx / D, d = idx - np * D, h = d / HALF, dd = d - h * HALF;
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) acc += sp[((int64_t)(q * 2 + h) * NP + np) * HALF + dd];
    part[(int64_t)blockIdx.x * NP * D + idx] = acc;
  }
}

// Sums the per-block partials: block = 32 columns x 16 row groups, each
// thread with four independent accumulators, combined in a fixed order
// through shared memory.
// np = 2 (dgamma, dbeta) or 3 (plus the column sums of the residual
// gradient, into rsum with its own accumulate flag).
__global__ void __launch_bounds__(512) ln_bwd_final_kernel(const float* __restrict__ part, int blocks, int D,
                                                           float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                           int accumulate, int np, float* __restrict__ rsum,
                                                           int rsum_accumulate) {
  pdl_wait();
  __shared__ float sm[16][33];
  const int d = blockIdx.x * 32 + threadIdx.x;
  const int64_t pd = (int64_t)np * D;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (d < pd) {
    int b = threadIdx.y;
    for (; b + 48 < blocks; b += 64) {
      s0 += part[(int64_t)b * pd + d];
      s1 += part[(int64_t)(b + 16) * pd + d];
      s2 += part[(int64_t)(b + 32) * pd + d];
      s3 += part[(int64_t)(b + 48) * pd + d];
    }
    for (; b < blocks; b += 16) s0 += part[(int64_t)b * pd + d];
  }
  sm[threadIdx.y][threadIdx.x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (threadIdx.y != 0 || d >= pd) return;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += sm[i][threadIdx.x];
  if (d >= 2 * D) {
    if (rsum) rsum[d - 2 * D] = rsum_accumulate ? rsum[d - 2 * D] + s : s;
    return;
  }
  float* dst = d < D ? (dgamma ? dgamma + d : nullptr) : (dbeta ? dbeta + (d - D) : nullptr);
  if (dst) *dst = accumulate ? *dst + s : s;
}

// ------------------------------------------------------------------ dropout
template <typename T>
__global__ void dropout_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = 1.f / (1.f - dd.p);
  const int64_t nb = (n + 3) >> 2;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
    const uint4 r = philox_block((uint64_t)b, dd.stream, step, dd.seed);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t i = b * 4 + j;
      if (i < n) y[i] = from_f32<T>(u01(pick(r, j)) >= dd.p ? to_f32(x[i]) * inv_keep : 0.f);
    }
  }
}

// ------------------------------------------------------------------ embedding
// out[i, :] = table[ids[i], :] (zeros for ids outside [0, V)).  One warp/row.
template <typename T>
__global__ void embed_fwd_kernel(const int32_t* __restrict__ ids, const T* __restrict__ table, T* __restrict__ out,
                                 int64_t n, int64_t V, int D) {
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int32_t id = ids[i];
  const bool ok = id >= 0 && id < V;
  T* o = out + i * D;
  const T* src = table + (int64_t)(ok ? id : 0) * D;
  if ((D * sizeof(T)) % 16 == 0 && ok) {
    const int nv = D * (int)sizeof(T) / 16;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* o4 = reinterpret_cast<uint4*>(o);
    for (int v = lane; v < nv; v += 32) o4[v] = s4[v];
  } else {
    for (int d = lane; d < D; d += 32) o[d] = ok ? src[d] : from_f32<T>(0.f);
  }
}

template <typename T>
__global__ void embed_bwd_kernel(const int32_t* __restrict__ ids, const T* __restrict__ dy, float* __restrict__ dtable,
                                 int64_t n, int64_t V, int D) {
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int32_t id = ids[i];
  if (id < 0 || id >= V) return;
  float* dst = dtable + (int64_t)id * D;
  const T* g = dy + i * D;
  for (int d = lane; d < D; d += 32) atomicAdd(dst + d, to_f32(g[d]));
}

inline unsigned grid1d(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

#define DLVK_DISPATCH_FB(dt, NAME, ...)                                         \
  do {                                                                          \
    if ((dt) == DType::F32) {                                                   \
      using T = float;                                                          \
      __VA_ARGS__;                                                              \
    } else if ((dt) == DType::BF16) {                                           \
      using T = __nv_bfloat16;                                                  \
      __VA_ARGS__;                                                              \
    } else {                                                                    \
      throw std::runtime_error(std::string("dlvk::") + NAME + ": unsupported dtype"); \
    }                                                                           \
  } while (0)

}  // namespace

namespace {
// Row chunks of the BatchNorm reductions: about four blocks per SM.
void bn_grid(int N, int C, int S, unsigned& groups, unsigned& chunks, int64_t& per) {
  if (S == 1) {
    groups = (unsigned)((C + BN_GROUP - 1) / BN_GROUP);
    const int64_t want = std::max<int64_t>(1, (4 * 148 + (int64_t)groups - 1) / groups);
    const int64_t ch = std::min<int64_t>(std::min<int64_t>(want, std::max<int64_t>(1, N / 8)), 1024);
    per = (N + ch - 1) / ch;
    chunks = (unsigned)((N + per - 1) / per);
  } else {
    groups = (unsigned)C;
    const int64_t cnt = (int64_t)N * S;
    const int64_t want = std::max<int64_t>(1, (4 * 148 + C - 1) / C);
    const int64_t ch = std::min<int64_t>(std::min<int64_t>(want, std::max<int64_t>(1, cnt / 2048)), 1024);
    per = (cnt + ch - 1) / ch;
    chunks = (unsigned)((cnt + per - 1) / per);
  }
}
bool al16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int64_t batchnorm_scratch_floats(int N, int C, int S) {
  unsigned groups, chunks;
  int64_t per;
  bn_grid(N, C, S, groups, chunks, per);
  return 7 * (int64_t)C + 2 * (int64_t)chunks * C;
}

void batchnorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s) {
  const BnCoef co = bn_coef(scratch, C);
  if (training) {
    unsigned groups, chunks;
    int64_t per;
    bn_grid(N, C, S, groups, chunks, per);
    const int vec = (S == 1 && C % 8 == 0 && al16p(x)) ? 1 : 0;
    DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_partial_kernel<T, 0><<<dim3(groups, chunks), 256, 0, s>>>(
        (const T*)x, nullptr, nullptr, nullptr, nullptr, nullptr, N, C, S, per, 0, DropoutDesc{}, vec, co.part));
    DLVK_POST_LAUNCH();
    DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_stats_finalize_kernel<T><<<(C + 31) / 32, 256, 0, s>>>(
        co.part, (int)chunks, (const T*)x, C, S, (int64_t)N * S, mean, rstd, run_mean, run_var, momentum, eps,
        gamma, beta, co));
  } else {
    bn_coef_kernel<<<(C + 255) / 256, 256, 0, s>>>(mean, rstd, gamma, beta, C, co);
  }
  DLVK_POST_LAUNCH();
  const int64_t total = (int64_t)N * C * S;
  if (total % 8 == 0 && al16p(x) && al16p(y) && al16p(scratch) && C % 4 == 0) {
    DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_apply_vec_kernel<T><<<grid1d(total / 8), 256, 0, s>>>(
        (const T*)x, co, (T*)y, total, C, S, relu ? 1 : 0, dd));
  } else {
    DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_apply_kernel<T><<<grid1d(total), 256, 0, s>>>(
        (const T*)x, co.scale, co.shift, (T*)y, total, C, S, relu ? 1 : 0, dd));
  }
  DLVK_POST_LAUNCH();
}

void batchnorm_bwd(DType dt, const void* x, const void* dy, const float* mean, const float* rstd, const float* gamma,
                   const float* beta, void* dx, float* dgamma, float* dbeta, bool accumulate, int N, int C, int S,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s) {
  const BnCoef co = bn_coef(scratch, C);
  unsigned groups, chunks;
  int64_t per;
  bn_grid(N, C, S, groups, chunks, per);
  const int vec = (S == 1 && C % 8 == 0 && al16p(x) && al16p(dy)) ? 1 : 0;
  DLVK_DISPATCH_FB(dt, "batchnorm_bwd", bn_partial_kernel<T, 1><<<dim3(groups, chunks), 256, 0, s>>>(
      (const T*)x, (const T*)dy, mean, rstd, gamma, beta, N, C, S, per, relu ? 1 : 0, dd, vec, co.part));
  DLVK_POST_LAUNCH();
  const float inv_count = 1.f / (float)((int64_t)N * S);
  bn_bwd_finalize_kernel<<<(C + 31) / 32, 256, 0, s>>>(co.part, (int)chunks, C, mean, rstd, gamma, beta, inv_count,
                                                        dgamma, dbeta, accumulate ? 1 : 0, co);
  DLVK_POST_LAUNCH();
  const int64_t total = (int64_t)N * C * S;
  if (total % 8 == 0 && al16p(x) && al16p(dy) && al16p(dx) && al16p(scratch) && C % 4 == 0) {
    DLVK_DISPATCH_FB(dt, "batchnorm_bwd", bn_bwd_apply_vec_kernel<T><<<grid1d(total / 8), 256, 0, s>>>(
        (const T*)x, (const T*)dy, co, (T*)dx, total, C, S, relu ? 1 : 0, dd));
  } else {
    DLVK_DISPATCH_FB(dt, "batchnorm_bwd", bn_bwd_apply_kernel<T><<<grid1d(total), 256, 0, s>>>(
        (const T*)x, (const T*)dy, co.A, co.B, co.D, co.shift, (T*)dx, total, C, S, relu ? 1 : 0, dd));
  }
  DLVK_POST_LAUNCH();
}

void layernorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   int64_t rows, int D, float eps, cudaStream_t s) {
  const int epv = dt == DType::F32 ? 4 : 8;
  const int nv = (D % (32 * epv) == 0) ? D / (32 * epv) : 0;
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                    reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
  if (al && (nv == 1 || nv == 2 || nv == 4)) {
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 148 * 2));
    const size_t smem = (size_t)2 * D * sizeof(float);
    DLVK_DISPATCH_FB(dt, "layernorm_fwd", {
      auto kern = nv == 1 ? ln_fwd_rows_kernel<T, 1, 4>
                          : (nv == 2 ? ln_fwd_rows_kernel<T, 2, 4> : ln_fwd_rows_kernel<T, 4, 2>);
      if (smem > 48 * 1024)
        DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      launch_pdl(kern, dim3(g), dim3(256), smem, s, (const T*)x, gamma, beta, (T*)y, mean, rstd, rows, D, eps);
    });
    DLVK_POST_LAUNCH();
    return;
  }
  if (al && (nv == 1 || nv == 2 || nv == 4 || nv == 8)) {
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, 148 * 4));
    DLVK_DISPATCH_FB(dt, "layernorm_fwd", {
      auto kern = nv == 1 ? ln_fwd_vec_kernel<T, 1>
                          : (nv == 2 ? ln_fwd_vec_kernel<T, 2> : (nv == 4 ? ln_fwd_vec_kernel<T, 4> : ln_fwd_vec_kernel<T, 8>));
      launch_pdl(kern, dim3(g), dim3(256), 0, s, (const T*)x, gamma, beta, (T*)y, mean, rstd, rows, D, eps);
    });
    DLVK_POST_LAUNCH();
    return;
  }
  const unsigned g = (unsigned)((rows + 7) / 8);
  DLVK_DISPATCH_FB(dt, "layernorm_fwd", ln_fwd_kernel<T><<<g, 256, 0, s>>>((const T*)x, gamma, beta, (T*)y, mean, rstd,
                                                                            rows, D, eps));
  DLVK_POST_LAUNCH();
}

int layernorm_bwd_blocks(int64_t rows) { return (int)std::max<int64_t>(1, std::min<int64_t>(148, (rows + 7) / 8)); }
// Per-block partials (up to three D-wide rows each) and, after them, the
// scratch of a column-sum pass over dres for the paths that do not fuse it.
int64_t layernorm_bwd_scratch_floats(int64_t rows, int D) {
  return (int64_t)layernorm_bwd_blocks(rows) * 3 * D + colsum_scratch_floats(rows, D);
}

void layernorm_bwd(DType dt, const void* x, const float* gamma, const float* mean, const float* rstd, const void* dy,
                   void* dx, float* dgamma, float* dbeta, bool accumulate, int64_t rows, int D, float* scratch,
                   cudaStream_t s, const void* dres, float* dres_colsum, bool dres_colsum_accumulate) {
  const int blocks = layernorm_bwd_blocks(rows);
  DLVK_CHECK(dres_colsum == nullptr || dres != nullptr, "layernorm_bwd: column sums of dres need dres");
  // Paths without the fused sums: a column-sum pass over dres.
  auto dres_sums = [&]() {
    if (!dres_colsum) return;
    float* cs = scratch + (int64_t)blocks * 3 * D;
    colsum(dt, DType::F32, dres, rows, D, 1.f, dres_colsum, dres_colsum_accumulate,
           colsum_scratch_floats(rows, D) > 0 ? cs : nullptr, s);
  };
  // Two warps per row (DLVK_LN_BWD_PAIR=0: one warp per row, the ring kernel below).
  static const bool pair_on = [] {
    const char* e = std::getenv("DLVK_LN_BWD_PAIR");
    return !(e && e[0] == '0');
  }();
  if (pair_on && dt == DType::BF16 && D % 512 == 0 && (D / 512 == 2 || D / 512 == 1)) {
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                      reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dres)) & 15) == 0;
    const int nvh = D / 512;
    const int nt = dres ? 3 : 2;
    const size_t ring = (size_t)16 * 3 * nt * nvh * 32 * 16;  // reused for the [16][NP][D/2] fp32 partials
    const size_t smem = ring + (size_t)D * 4 + 16 * 3 * 2 * 4 + 8 * 2 * 2 * 8;  // ring | gamma | row stats | exchange
    if (al && ring >= (size_t)16 * (dres ? 3 : 2) * (D / 2) * 4 && smem <= 200 * 1024) {
      auto launch = [&](auto kern) {
        DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        launch_pdl(kern, dim3(blocks), dim3(512), smem, s, (const __nv_bfloat16*)x, gamma, mean, rstd,
                   (const __nv_bfloat16*)dy, (__nv_bfloat16*)dx, scratch, rows, D, (const __nv_bfloat16*)dres);
      };
      if (dres) {
        if (nvh == 2) launch(ln_bwd_pair_kernel<2, true>);
        else launch(ln_bwd_pair_kernel<1, true>);
      } else {
        if (nvh == 2) launch(ln_bwd_pair_kernel<2, false>);
        else launch(ln_bwd_pair_kernel<1, false>);
      }
      DLVK_POST_LAUNCH();
      const int np = dres ? 3 : 2;
      launch_pdl(ln_bwd_final_kernel, dim3((np * D + 31) / 32), dim3(32, 16), 0, s, (const float*)scratch, blocks, D,
                 dgamma, dbeta, accumulate ? 1 : 0, np, dres_colsum, dres_colsum_accumulate ? 1 : 0);
      DLVK_POST_LAUNCH();
      return;
    }
  }
  if (dt == DType::BF16 && D % 256 == 0 && (D / 256 == 4 || D / 256 == 2 || D / 256 == 1)) {
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                      reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dres)) & 15) == 0;
    const int nv = D / 256;
    const int nt = dres ? 3 : 2;
    const size_t ring = (size_t)8 * 3 * nt * nv * 32 * 16;  // reused for the [8][2D or 3D] fp32 partials
    const size_t smem = ring + (size_t)D * 4;
    if (al && ring >= (size_t)8 * (dres ? 3 : 2) * D * 4 && smem <= 200 * 1024) {
      auto launch = [&](auto kern) {
        DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        launch_pdl(kern, dim3(blocks), dim3(256), smem, s, (const __nv_bfloat16*)x, gamma, mean, rstd,
                   (const __nv_bfloat16*)dy, (__nv_bfloat16*)dx, scratch, rows, D, (const __nv_bfloat16*)dres);
      };
      if (dres) {
        if (nv == 4) launch(ln_bwd_ring_kernel<4, true>);
        else if (nv == 2) launch(ln_bwd_ring_kernel<2, true>);
        else launch(ln_bwd_ring_kernel<1, true>);
      } else {
        if (nv == 4) launch(ln_bwd_ring_kernel<4, false>);
        else if (nv == 2) launch(ln_bwd_ring_kernel<2, false>);
        else launch(ln_bwd_ring_kernel<1, false>);
      }
      DLVK_POST_LAUNCH();
      const int np = dres ? 3 : 2;
      launch_pdl(ln_bwd_final_kernel, dim3((np * D + 31) / 32), dim3(32, 16), 0, s, (const float*)scratch, blocks, D,
                 dgamma, dbeta, accumulate ? 1 : 0, np, dres_colsum, dres_colsum_accumulate ? 1 : 0);
      DLVK_POST_LAUNCH();
      return;
    }
  }
  {
    // Register-resident path: D a multiple of 32 lanes x 16-byte vectors.
    const int epv = dt == DType::F32 ? 4 : 8;
    const int nv = (D % (32 * epv) == 0) ? D / (32 * epv) : 0;
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                      reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dres)) & 15) == 0;
    const size_t smem = (size_t)(8 * 2 + 1) * D * sizeof(float);
    if (al && (nv == 1 || nv == 2 || nv == 4) && smem <= 200 * 1024) {
      DLVK_DISPATCH_FB(dt, "layernorm_bwd", {
        auto kern = nv == 1 ? ln_bwd_warp_kernel<T, 1> : (nv == 2 ? ln_bwd_warp_kernel<T, 2> : ln_bwd_warp_kernel<T, 4>);
        if (smem > 48 * 1024)
          DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        kern<<<blocks, 256, smem, s>>>((const T*)x, gamma, mean, rstd, (const T*)dy, (T*)dx, scratch, rows, D,
                                       (const T*)dres);
      });
      DLVK_POST_LAUNCH();
      ln_bwd_final_kernel<<<(2 * D + 31) / 32, dim3(32, 16), 0, s>>>(scratch, blocks, D, dgamma, dbeta, accumulate ? 1 : 0,
                                                                    2, nullptr, 0);
      DLVK_POST_LAUNCH();
      dres_sums();
      return;
    }
  }
  int warps = 8;
  while (warps > 1 && (size_t)warps * 2 * D * sizeof(float) > 96 * 1024) warps >>= 1;
  const size_t smem = (size_t)warps * 2 * D * sizeof(float);
  DLVK_CHECK(smem <= 200 * 1024, "layernorm_bwd: feature dimension too large");
  DLVK_DISPATCH_FB(dt, "layernorm_bwd", {
    if (smem > 48 * 1024)
      DLVK_CUDA_CHECK(cudaFuncSetAttribute(ln_bwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ln_bwd_kernel<T><<<blocks, warps * 32, smem, s>>>((const T*)x, gamma, mean, rstd, (const T*)dy, (T*)dx, scratch,
                                                      rows, D, (const T*)dres);
  });
  DLVK_POST_LAUNCH();
  ln_bwd_final_kernel<<<(2 * D + 31) / 32, dim3(32, 16), 0, s>>>(scratch, blocks, D, dgamma, dbeta, accumulate ? 1 : 0,
                                                                2, nullptr, 0);
  DLVK_POST_LAUNCH();
  dres_sums();
}

void dropout(DType dt, const void* x, void* y, int64_t n, const DropoutDesc& dd, cudaStream_t s) {
  if (n == 0) return;
  DLVK_DISPATCH_FB(dt, "dropout", dropout_kernel<T><<<grid1d((n + 3) / 4), 256, 0, s>>>((const T*)x, (T*)y, n, dd));
  DLVK_POST_LAUNCH();
}

void embedding_fwd(DType dt, const int32_t* ids, const void* table, void* out, int64_t n, int64_t V, int D,
                   cudaStream_t s) {
  if (n == 0) return;
  DLVK_DISPATCH_FB(dt, "embedding_fwd", embed_fwd_kernel<T><<<(unsigned)((n + 7) / 8), 256, 0, s>>>(
      ids, (const T*)table, (T*)out, n, V, D));
  DLVK_POST_LAUNCH();
}

void embedding_bwd(DType dt, const int32_t* ids, const void* dy, float* dtable, int64_t n, int64_t V, int D,
                   cudaStream_t s) {
  if (n == 0) return;
  DLVK_DISPATCH_FB(dt, "embedding_bwd", embed_bwd_kernel<T><<<(unsigned)((n + 7) / 8), 256, 0, s>>>(
      ids, (const T*)dy, dtable, n, V, D));
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
