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
// Column statistics of x viewed as [N, C, S]; one thread block of 256 threads
// per group of channels.  S == 1 (BatchNorm1D): 64 channels per block, rows
// strided over 4 thread rows.  S > 1: one block per channel.
// Uses shifted sums (shift = first element) for a stable variance.
template <typename T>
__global__ void bn_stats_kernel(const T* __restrict__ x, int N, int C, int S, float* __restrict__ mean,
                                float* __restrict__ rstd, float* __restrict__ run_mean, float* __restrict__ run_var,
                                float momentum, float eps) {
  if (S == 1) {
    __shared__ float s1[4][64], s2[4][64];
    const int cl = threadIdx.x & 63, rg = threadIdx.x >> 6;
    const int c = blockIdx.x * 64 + cl;
    float a = 0.f, b = 0.f, shift = 0.f;
    if (c < C) {
      shift = to_f32(x[c]);
      for (int n = rg; n < N; n += 4) {
        const float v = to_f32(x[(int64_t)n * C + c]) - shift;
        a += v;
        b += v * v;
      }
    }
    s1[rg][cl] = a;
    s2[rg][cl] = b;
    __syncthreads();
    if (rg == 0 && c < C) {
      a = s1[0][cl] + s1[1][cl] + s1[2][cl] + s1[3][cl];
      b = s2[0][cl] + s2[1][cl] + s2[2][cl] + s2[3][cl];
      const float m1 = a / N;
      const float var = fmaxf(b / N - m1 * m1, 0.f);
      const float mu = m1 + shift;
      mean[c] = mu;
      rstd[c] = rsqrtf(var + eps);
      if (run_mean) run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
      if (run_var) run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
    }
  } else {
    __shared__ float sm[32];
    const int c = blockIdx.x;
    const float shift = to_f32(x[(int64_t)c * S]);
    float a = 0.f, b = 0.f;
    const int64_t cnt = (int64_t)N * S;
    for (int64_t i = threadIdx.x; i < cnt; i += blockDim.x) {
      const int64_t n = i / S, sp = i - n * S;
      const float v = to_f32(x[(n * C + c) * S + sp]) - shift;
      a += v;
      b += v * v;
    }
    a = block_sum(a, sm);
    b = block_sum(b, sm);
    if (threadIdx.x == 0) {
      const float m1 = a / cnt;
      const float var = fmaxf(b / cnt - m1 * m1, 0.f);
      const float mu = m1 + shift;
      mean[c] = mu;
      rstd[c] = rsqrtf(var + eps);
      if (run_mean) run_mean[c] = (1.f - momentum) * run_mean[c] + momentum * mu;
      if (run_var) run_var[c] = (1.f - momentum) * run_var[c] + momentum * var;
    }
  }
}

// y = dropout(relu(gamma * (x - mean) * rstd + beta))
template <typename T>
__global__ void bn_apply_kernel(const T* __restrict__ x, const float* __restrict__ mean, const float* __restrict__ rstd,
                                const float* __restrict__ gamma, const float* __restrict__ beta, T* __restrict__ y,
                                int64_t total, int C, int S, int relu, DropoutDesc dd) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / S) % C);
    float v = (to_f32(x[i]) - mean[c]) * rstd[c] * (gamma ? gamma[c] : 1.f) + (beta ? beta[c] : 0.f);
    if (relu) v = fmaxf(v, 0.f);
    if (dd.p > 0.f) v = keep_elem(i, dd, step) ? v * inv_keep : 0.f;
    y[i] = from_f32<T>(v);
  }
}

// Gradient w.r.t. the normalised pre-activation, undoing dropout and ReLU.
template <typename T>
__device__ __forceinline__ float bn_upstream(const T* dy, const T* x, int64_t i, int c, const float* mean,
                                             const float* rstd, const float* gamma, const float* beta, int relu,
                                             const DropoutDesc& dd, uint32_t step, float inv_keep, float& xhat) {
  xhat = (to_f32(x[i]) - mean[c]) * rstd[c];
  float g = to_f32(dy[i]);
  if (dd.p > 0.f) g = keep_elem(i, dd, step) ? g * inv_keep : 0.f;
  if (relu) {
    const float pre = xhat * (gamma ? gamma[c] : 1.f) + (beta ? beta[c] : 0.f);
    if (!(pre > 0.f)) g = 0.f;
  }
  return g;
}

// Per-channel sums: sg[c] = sum g, sgx[c] = sum g * xhat.  Same layouts as
// bn_stats_kernel.  Writes dbeta/dgamma (optionally accumulating).
template <typename T>
__global__ void bn_bwd_reduce_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ mean,
                                     const float* __restrict__ rstd, const float* __restrict__ gamma,
                                     const float* __restrict__ beta, int N, int C, int S, int relu, DropoutDesc dd,
                                     float* __restrict__ sg_out, float* __restrict__ sgx_out,
                                     float* __restrict__ dgamma, float* __restrict__ dbeta, int accumulate) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  float a = 0.f, b = 0.f;
  int c;
  if (S == 1) {
    __shared__ float s1[4][64], s2[4][64];
    const int cl = threadIdx.x & 63, rg = threadIdx.x >> 6;
    c = blockIdx.x * 64 + cl;
    if (c < C) {
      for (int n = rg; n < N; n += 4) {
        float xh;
        const int64_t i = (int64_t)n * C + c;
        const float g = bn_upstream(dy, x, i, c, mean, rstd, gamma, beta, relu, dd, step, inv_keep, xh);
        a += g;
        b += g * xh;
      }
    }
    s1[rg][cl] = a;
    s2[rg][cl] = b;
    __syncthreads();
    if (rg != 0 || c >= C) return;
    a = s1[0][cl] + s1[1][cl] + s1[2][cl] + s1[3][cl];
    b = s2[0][cl] + s2[1][cl] + s2[2][cl] + s2[3][cl];
  } else {
    __shared__ float sm[32];
    c = blockIdx.x;
    const int64_t cnt = (int64_t)N * S;
    for (int64_t k = threadIdx.x; k < cnt; k += blockDim.x) {
      const int64_t n = k / S, sp = k - n * S;
      const int64_t i = (n * C + c) * S + sp;
      float xh;
      const float g = bn_upstream(dy, x, i, c, mean, rstd, gamma, beta, relu, dd, step, inv_keep, xh);
      a += g;
      b += g * xh;
    }
    a = block_sum(a, sm);
    b = block_sum(b, sm);
    if (threadIdx.x != 0) return;
  }
  sg_out[c] = a;
  sgx_out[c] = b;
  if (dbeta) dbeta[c] = accumulate ? dbeta[c] + a : a;
  if (dgamma) dgamma[c] = accumulate ? dgamma[c] + b : b;
}

// dx = gamma * rstd * (g - sg / M - xhat * sgx / M)
template <typename T>
__global__ void bn_bwd_apply_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ mean,
                                    const float* __restrict__ rstd, const float* __restrict__ gamma,
                                    const float* __restrict__ beta, const float* __restrict__ sg,
                                    const float* __restrict__ sgx, T* __restrict__ dx, int64_t total, int C, int S,
                                    int relu, DropoutDesc dd, float inv_count) {
  const uint32_t step = read_step(dd);
  const float inv_keep = dd.p > 0.f ? 1.f / (1.f - dd.p) : 1.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)((i / S) % C);
    float xh;
    const float g = bn_upstream(dy, x, i, c, mean, rstd, gamma, beta, relu, dd, step, inv_keep, xh);
    const float v = (gamma ? gamma[c] : 1.f) * rstd[c] * (g - sg[c] * inv_count - xh * sgx[c] * inv_count);
    dx[i] = from_f32<T>(v);
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
  constexpr int EPV = 8, RING = 3, NT = RES ? 3 : 2, RV = NV * 32;  // 16-byte vectors per tensor row
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
  float adg[NV][EPV], adb[NV][EPV];
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) adg[i][k] = adb[i][k] = 0.f;
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
        const float gg = g * sgam[(lane + 32 * i) * EPV + k];
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
        float v = rs * (__bfloat162float(eg[k]) * sgam[(lane + 32 * i) * EPV + k] - a - xh * bb);
        if (RES) v += __bfloat162float(er[k]);
        eo[k] = __float2bfloat16_rn(v);
      }
      reinterpret_cast<uint4*>(dx + r * D)[lane + 32 * i] = o;
    }
    issue(r + RING * step, slot);  // this lane has read its vectors of the slot
    slot = slot + 1 == RING ? 0 : slot + 1;
  }
  sm100::cp_async_wait<0>();
  __syncthreads();
  float* sp = reinterpret_cast<float*>(sring);  // the ring is free: [8][2*D] partials
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
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += sp[(int64_t)i * 2 * D + d];
    part[(int64_t)blockIdx.x * 2 * D + d] = acc;
  }
}

// Sums the per-block partials: block = 32 columns x 16 row groups, each
// thread with four independent accumulators, combined in a fixed order
// through shared memory.
__global__ void __launch_bounds__(512) ln_bwd_final_kernel(const float* __restrict__ part, int blocks, int D,
                                                           float* __restrict__ dgamma, float* __restrict__ dbeta,
                                                           int accumulate) {
  pdl_wait();
  __shared__ float sm[16][33];
  const int d = blockIdx.x * 32 + threadIdx.x;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (d < 2 * D) {
    int b = threadIdx.y;
    for (; b + 48 < blocks; b += 64) {
      s0 += part[(int64_t)b * 2 * D + d];
      s1 += part[(int64_t)(b + 16) * 2 * D + d];
      s2 += part[(int64_t)(b + 32) * 2 * D + d];
      s3 += part[(int64_t)(b + 48) * 2 * D + d];
    }
    for (; b < blocks; b += 16) s0 += part[(int64_t)b * 2 * D + d];
  }
  sm[threadIdx.y][threadIdx.x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (threadIdx.y != 0 || d >= 2 * D) return;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) s += sm[i][threadIdx.x];
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

void batchnorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   float* run_mean, float* run_var, int N, int C, int S, float momentum, float eps, bool training,
                   bool relu, const DropoutDesc& dd, cudaStream_t s) {
  if (training) {
    const unsigned g = S == 1 ? (unsigned)((C + 63) / 64) : (unsigned)C;
    DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_stats_kernel<T><<<g, 256, 0, s>>>(
        (const T*)x, N, C, S, mean, rstd, run_mean, run_var, momentum, eps));
    DLVK_POST_LAUNCH();
  }
  const int64_t total = (int64_t)N * C * S;
  DLVK_DISPATCH_FB(dt, "batchnorm_fwd", bn_apply_kernel<T><<<grid1d(total), 256, 0, s>>>(
      (const T*)x, mean, rstd, gamma, beta, (T*)y, total, C, S, relu ? 1 : 0, dd));
  DLVK_POST_LAUNCH();
}

void batchnorm_bwd(DType dt, const void* x, const void* dy, const float* mean, const float* rstd, const float* gamma,
                   const float* beta, void* dx, float* dgamma, float* dbeta, bool accumulate, int N, int C, int S,
                   bool relu, const DropoutDesc& dd, float* scratch, cudaStream_t s) {
  float* sg = scratch;
  float* sgx = scratch + C;
  const unsigned g = S == 1 ? (unsigned)((C + 63) / 64) : (unsigned)C;
  DLVK_DISPATCH_FB(dt, "batchnorm_bwd", bn_bwd_reduce_kernel<T><<<g, 256, 0, s>>>(
      (const T*)x, (const T*)dy, mean, rstd, gamma, beta, N, C, S, relu ? 1 : 0, dd, sg, sgx, dgamma, dbeta,
      accumulate ? 1 : 0));
  DLVK_POST_LAUNCH();
  const int64_t total = (int64_t)N * C * S;
  DLVK_DISPATCH_FB(dt, "batchnorm_bwd", bn_bwd_apply_kernel<T><<<grid1d(total), 256, 0, s>>>(
      (const T*)x, (const T*)dy, mean, rstd, gamma, beta, sg, sgx, (T*)dx, total, C, S, relu ? 1 : 0, dd,
      1.f / (float)((int64_t)N * S)));
  DLVK_POST_LAUNCH();
}

void layernorm_fwd(DType dt, const void* x, const float* gamma, const float* beta, void* y, float* mean, float* rstd,
                   int64_t rows, int D, float eps, cudaStream_t s) {
  const int epv = dt == DType::F32 ? 4 : 8;
  const int nv = (D % (32 * epv) == 0) ? D / (32 * epv) : 0;
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                    reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
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
int64_t layernorm_bwd_scratch_floats(int64_t rows, int D) { return (int64_t)layernorm_bwd_blocks(rows) * 2 * D; }

void layernorm_bwd(DType dt, const void* x, const float* gamma, const float* mean, const float* rstd, const void* dy,
                   void* dx, float* dgamma, float* dbeta, bool accumulate, int64_t rows, int D, float* scratch,
                   cudaStream_t s, const void* dres) {
  const int blocks = layernorm_bwd_blocks(rows);
  if (dt == DType::BF16 && D % 256 == 0 && (D / 256 == 4 || D / 256 == 2 || D / 256 == 1)) {
    const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                      reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(dres)) & 15) == 0;
    const int nv = D / 256;
    const int nt = dres ? 3 : 2;
    const size_t ring = (size_t)8 * 3 * nt * nv * 32 * 16;  // reused for the [8][2D] fp32 partials
    const size_t smem = ring + (size_t)D * 4;
    if (al && ring >= (size_t)8 * 2 * D * 4 && smem <= 200 * 1024) {
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
      launch_pdl(ln_bwd_final_kernel, dim3((2 * D + 31) / 32), dim3(32, 16), 0, s, (const float*)scratch, blocks, D,
                 dgamma, dbeta, accumulate ? 1 : 0);
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
      ln_bwd_final_kernel<<<(2 * D + 31) / 32, dim3(32, 16), 0, s>>>(scratch, blocks, D, dgamma, dbeta, accumulate ? 1 : 0);
      DLVK_POST_LAUNCH();
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
  ln_bwd_final_kernel<<<(2 * D + 31) / 32, dim3(32, 16), 0, s>>>(scratch, blocks, D, dgamma, dbeta, accumulate ? 1 : 0);
  DLVK_POST_LAUNCH();
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
