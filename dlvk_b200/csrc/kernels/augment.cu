// Batched image transforms for the data pipeline, on the device.
//
// Reference: data transforms (src/data/transforms.cpp:26-680) run one
// sample at a time on the host (download, loop, upload).  Here each
// transform is one kernel over a whole [N, C, H, W] fp32 batch already in
// HBM, with per-sample random parameters drawn by the caller:
//
//  * affine_sample: out(n,c,y,x) = in(n,c, T_n(x,y)) where T_n is a 2x3
//    map from output to input coordinates -- flips, crops (with zero
//    padding), rotation about the centre, zoom and resize are all such
//    maps.  Modes: nearest with floor (crop/scale/resize), nearest with
//    round-half-away (rotation, transforms.cpp:256-300), bilinear with
//    the lower/left neighbour clamped to the image and the upper/right one
//    clamped to the last row/column (Resize, transforms.cpp:592-660).
//    Samples outside the image read `fill`.
//  * per_sample_affine_stats: one CTA per sample computes mean / std /
//    min / max over C*H*W and applies y = clamp(a_n * x + b_n(stats)) for
//    contrast (mean + c (x - mean)), standardisation ((x - mean) / std)
//    and min-max scaling (transforms.cpp:69-125, 476-505).
//  * channel_affine: y = (x - mean[c]) * inv_std[c] (Normalize), plus a
//    per-sample additive term and clamp (brightness, transforms.cpp:452-475).
//  * gaussian_noise: y = x + sigma * N(0,1) from Philox4x32-10 keyed by a
//    seed, Box-Muller on two uniforms (RandomNoise, transforms.cpp:430-450).
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

__global__ void affine_sample_kernel(const float* __restrict__ x, float* __restrict__ y, int C, int H, int W,
                                     int OH, int OW, const float* __restrict__ theta, int mode, float fill) {
  const int n = blockIdx.z;
  const int64_t plane_out = (int64_t)OH * OW;
  const float* t = theta + 6 * n;
  const float a = t[0], b = t[1], c0 = t[2], d = t[3], e = t[4], f = t[5];
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < plane_out;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int oy = (int)(p / OW), ox = (int)(p % OW);
    const float sx = a * ox + b * oy + c0;
    const float sy = d * ox + e * oy + f;
    for (int c = blockIdx.y; c < C; c += gridDim.y) {
      const float* src = x + ((int64_t)n * C + c) * H * W;
      float v = fill;
      if (mode == 2) {  // bilinear
        const float fx = floorf(sx), fy = floorf(sy);
        const int x1 = (int)fx, y1 = (int)fy;
        if (x1 >= 0 && x1 < W && y1 >= 0 && y1 < H) {
          const int x2 = min(x1 + 1, W - 1), y2 = min(y1 + 1, H - 1);
          const float dx = sx - fx, dy = sy - fy;
          v = src[y1 * W + x1] * (1.f - dy) * (1.f - dx) + src[y1 * W + x2] * (1.f - dy) * dx +
              src[y2 * W + x1] * dy * (1.f - dx) + src[y2 * W + x2] * dy * dx;
        }
      } else {
        const int ix = mode == 1 ? (int)roundf(sx) : (int)floorf(sx);
        const int iy = mode == 1 ? (int)roundf(sy) : (int)floorf(sy);
        if (ix >= 0 && ix < W && iy >= 0 && iy < H) v = src[iy * W + ix];
      }
      y[((int64_t)n * C + c) * plane_out + p] = v;
    }
  }
}

// kind 0: contrast  y = mean + p0 * (x - mean)
// kind 1: standardise y = (x - mean) / std  (unchanged if std <= 1e-8)
// kind 2: min-max   y = p0 + (x - min) * (p1 - p0) / (max - min)  (unchanged if range <= 1e-8)
__global__ void per_sample_stats_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t len, int kind,
                                        const float* __restrict__ params, int clamp01) {
  __shared__ float sm[32];
  __shared__ float stats[4];
  const int n = blockIdx.x;
  const float* xs = x + (int64_t)n * len;
  float* ys = y + (int64_t)n * len;
  float s = 0.f, mn = INFINITY, mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
    const float v = xs[i];
    s += v;
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  s = block_sum(s, sm);
  mn = -block_max(-mn, sm);
  mx = block_max(mx, sm);
  const float mean = s / (float)len;
  float q = 0.f;
  if (kind == 1) {
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
      const float dv = xs[i] - mean;
      q += dv * dv;
    }
    q = block_sum(q, sm);
  }
  if (threadIdx.x == 0) {
    stats[0] = mean;
    stats[1] = sqrtf(q / (float)len);
    stats[2] = mn;
    stats[3] = mx;
  }
  __syncthreads();
  const float p0 = params ? params[2 * n] : 0.f, p1 = params ? params[2 * n + 1] : 0.f;
  float A = 1.f, B = 0.f;
  if (kind == 0) {
    A = p0;
    B = stats[0] * (1.f - p0);
  } else if (kind == 1) {
    if (stats[1] > 1e-8f) {
      A = 1.f / stats[1];
      B = -stats[0] * A;
    }
  } else {
    const float range = stats[3] - stats[2];
    if (range > 1e-8f) {
      A = (p1 - p0) / range;
      B = p0 - stats[2] * A;
    }
  }
  for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
    float v = A * xs[i] + B;
    if (clamp01) v = fminf(fmaxf(v, 0.f), 1.f);
    ys[i] = v;
  }
}

__global__ void channel_affine_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t N, int C,
                                      int64_t HW, const float* __restrict__ mean, const float* __restrict__ inv_std,
                                      const float* __restrict__ sample_add, int clamp01) {
  const int64_t total = N * C * HW;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t nc = i / HW;
    const int c = (int)(nc % C);
    float v = x[i];
    if (sample_add) v += sample_add[nc / C];
    if (mean) v = (v - mean[c]) * inv_std[c];
    if (clamp01) v = fminf(fmaxf(v, 0.f), 1.f);
    y[i] = v;
  }
}

__global__ void gaussian_noise_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n, float sigma,
                                      uint32_t seed_lo, uint32_t seed_hi, uint32_t stream) {
  const int64_t groups = (n + 3) / 4;
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < groups; g += (int64_t)gridDim.x * blockDim.x) {
    const uint4 r = philox4x32_10(make_uint4((uint32_t)g, (uint32_t)(g >> 32), stream, 0x6e6f6973u),
                                  make_uint2(seed_lo, seed_hi));
    // Box-Muller: two normals from each pair of uniforms
    const float u0 = fmaxf(u01(r.x), 1e-12f), u1 = u01(r.y), u2 = fmaxf(u01(r.z), 1e-12f), u3 = u01(r.w);
    const float r0 = sqrtf(-2.f * logf(u0)), r1 = sqrtf(-2.f * logf(u2));
    float nz[4];
    sincospif(2.f * u1, &nz[1], &nz[0]);
    sincospif(2.f * u3, &nz[3], &nz[2]);
    nz[0] *= r0;
    nz[1] *= r0;
    nz[2] *= r1;
    nz[3] *= r1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t i = g * 4 + k;
      if (i < n) y[i] = x[i] + sigma * nz[k];
    }
  }
}

int blocks_for(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8)); }

}  // namespace

void image_affine_sample(const float* x, float* y, int N, int C, int H, int W, int OH, int OW, const float* theta,
                         int mode, float fill, cudaStream_t s) {
  if (N == 0) return;
  const int64_t plane = (int64_t)OH * OW;
  dim3 grid((unsigned)std::max<int64_t>(1, std::min<int64_t>((plane + 255) / 256, 64)), (unsigned)std::min(C, 4),
            (unsigned)N);
  affine_sample_kernel<<<grid, 256, 0, s>>>(x, y, C, H, W, OH, OW, theta, mode, fill);
  DLVK_POST_LAUNCH();
}

void image_per_sample_stats(const float* x, float* y, int64_t N, int64_t len, int kind, const float* params,
                            bool clamp01, cudaStream_t s) {
  if (N == 0) return;
  per_sample_stats_kernel<<<(unsigned)N, 512, 0, s>>>(x, y, len, kind, params, clamp01 ? 1 : 0);
  DLVK_POST_LAUNCH();
}

void image_channel_affine(const float* x, float* y, int64_t N, int C, int64_t HW, const float* mean,
                          const float* inv_std, const float* sample_add, bool clamp01, cudaStream_t s) {
  const int64_t total = N * C * HW;
  if (total == 0) return;
  channel_affine_kernel<<<blocks_for(total), 256, 0, s>>>(x, y, N, C, HW, mean, inv_std, sample_add,
                                                          clamp01 ? 1 : 0);
  DLVK_POST_LAUNCH();
}

void image_gaussian_noise(const float* x, float* y, int64_t n, float sigma, uint64_t seed, uint32_t stream,
                          cudaStream_t s) {
  if (n == 0) return;
  gaussian_noise_kernel<<<blocks_for((n + 3) / 4), 256, 0, s>>>(x, y, n, sigma, (uint32_t)seed,
                                                                (uint32_t)(seed >> 32), stream);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
