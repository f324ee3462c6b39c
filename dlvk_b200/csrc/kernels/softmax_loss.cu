// Softmax, fused softmax + cross-entropy (forward and backward in one pass),
// and the MSE / BCE losses.
//
// Reference: shaders/softmax.comp:23-67 (three dispatches: row max, exp+sum,
// divide), shaders/cross_entropy_{forward,backward}.comp, shaders/mse_*.comp,
// shaders/binary_cross_entropy_*.comp; host in src/loss/loss_functions.cpp
// (CPU CE = -sum t*log(p+1e-8)/B, grad (p - t)/B at :127-160).
// Here softmax is one kernel per row block, and softmax + CE produces the
// per-row loss and dlogits = (softmax - target) * scale from the logits in a
// single launch (the reference's softmax-backward-is-identity convention,
// src/layers/activation.cpp:71-75, is only correct in this fused form).
#include <type_traits>

#include <cstdlib>

#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/sm100.h"

namespace dlvk {
namespace {

// Merge two (max, sum-of-exp) pairs.
__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s = s + s2 * expf(m2 - m);
  }
}

template <int THREADS>
__device__ __forceinline__ void block_ms(float& m, float& s) {
  __shared__ float sm_m[32], sm_s[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ms_merge(m, s, m2, s2);
  }
  if (THREADS > 32) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) { sm_m[wid] = m; sm_s[wid] = s; }
    __syncthreads();
    m = -INFINITY;
    s = 0.f;
    for (int i = 0; i < THREADS / 32; ++i) ms_merge(m, s, sm_m[i], sm_s[i]);
  }
}

template <int THREADS>
__device__ __forceinline__ float block_sum_t(float v) {
  __shared__ float sm[32];
  v = warp_sum(v);
  if (THREADS > 32) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sm[wid] = v;
    __syncthreads();
    v = 0.f;
    for (int i = 0; i < THREADS / 32; ++i) v += sm[i];
  }
  return v;
}

// One CTA (THREADS threads) per row.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_rows_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                               int64_t cols, bool log_out) {
  const int64_t r = blockIdx.x;
  const T* xr = x + r * cols;
  T* yr = y + r * cols;
  float m = -INFINITY, s = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += THREADS) {
    const float v = to_f32(xr[c]);
    ms_merge(m, s, v, 1.f);
  }
  block_ms<THREADS>(m, s);
  const float inv = 1.f / s, lse = m + logf(s);
  for (int64_t c = threadIdx.x; c < cols; c += THREADS) {
    const float v = to_f32(xr[c]);
    yr[c] = from_f32<T>(log_out ? v - lse : expf(v - m) * inv);
  }
}

// dx = y * (dy - sum(dy * y))  (standard softmax Jacobian-vector product)
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_bwd_kernel(const T* __restrict__ y, const T* __restrict__ dy,
                                                              T* __restrict__ dx, int64_t cols) {
  const int64_t r = blockIdx.x;
  float acc = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += THREADS) acc += to_f32(y[r * cols + c]) * to_f32(dy[r * cols + c]);
  acc = block_sum_t<THREADS>(acc);
  for (int64_t c = threadIdx.x; c < cols; c += THREADS) {
    const float yy = to_f32(y[r * cols + c]);
    dx[r * cols + c] = from_f32<T>(yy * (to_f32(dy[r * cols + c]) - acc));
  }
}

// Fused softmax + cross-entropy.  Targets are either class ids (labels, -1 =
// ignored row) or a dense probability matrix `probs` [rows, cols].
// loss_rows[r] = -sum_c t_c * log_softmax(x)_c
// dlogits[r, c] = (softmax(x)_c - t_c) * grad_scale   (may alias x)
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) softmax_ce_kernel(const T* x, const int* __restrict__ labels,
                                                             const float* __restrict__ probs,
                                                             float* __restrict__ loss_rows, T* dlogits,
                                                             int64_t cols, float grad_scale) {
  constexpr int EPV = 16 / sizeof(T);
  const int64_t r = blockIdx.x;
  const T* xr = x + r * cols;
  // 16-byte vector path when the row is a whole number of aligned vectors.
  const bool vec = (cols % EPV) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0 &&
                   (!dlogits || (reinterpret_cast<uintptr_t>(dlogits + r * cols) & 15) == 0);
  float m = -INFINITY, s = 0.f;
  if (vec) {
    for (int64_t c8 = threadIdx.x; c8 < cols / EPV; c8 += THREADS) {
      const uint4 u = reinterpret_cast<const uint4*>(xr)[c8];
      const T* e = reinterpret_cast<const T*>(&u);
      float v[EPV], lm = -INFINITY;
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        v[k] = to_f32(e[k]);
        lm = fmaxf(lm, v[k]);
      }
      if (lm > m) {
        s = (m == -INFINITY) ? 0.f : s * expf(m - lm);
        m = lm;
      }
#pragma unroll
      for (int k = 0; k < EPV; ++k) s += expf(v[k] - m);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) ms_merge(m, s, to_f32(xr[c]), 1.f);
  }
  block_ms<THREADS>(m, s);
  const float lse = m + logf(s), inv = 1.f / s;
  const int label = labels ? labels[r] : -2;
  if (dlogits && vec && labels) {
    // Loss first (thread 0 reads the label logit), then the gradient pass.
    float loss = 0.f;
    if (label >= 0 && label < cols && threadIdx.x == 0) loss = lse - to_f32(xr[label]);
    loss = block_sum_t<THREADS>(loss);
    if (threadIdx.x == 0 && loss_rows) loss_rows[r] = label < 0 ? 0.f : loss;
    T* dr = dlogits + r * cols;
    const float gs = label < 0 ? 0.f : grad_scale;
    for (int64_t c8 = threadIdx.x; c8 < cols / EPV; c8 += THREADS) {
      const uint4 u = reinterpret_cast<const uint4*>(xr)[c8];
      const T* e = reinterpret_cast<const T*>(&u);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int k = 0; k < EPV; ++k) {
        const int64_t c = c8 * EPV + k;
        const float p = expf(to_f32(e[k]) - m) * inv;
        oe[k] = from_f32<T>((p - (c == label ? 1.f : 0.f)) * gs);
      }
      reinterpret_cast<uint4*>(dr)[c8] = o;
    }
    return;
  }
  float loss = 0.f;
  if (labels) {
    if (label >= 0 && label < cols && threadIdx.x == 0) loss = lse - to_f32(xr[label]);
  } else {
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) {
      const float t = probs[r * cols + c];
      if (t != 0.f) acc += t * (lse - to_f32(xr[c]));
    }
    loss = acc;
  }
  loss = block_sum_t<THREADS>(loss);
  if (threadIdx.x == 0 && loss_rows) loss_rows[r] = (labels && label < 0) ? 0.f : loss;
  if (dlogits) {
    T* dr = dlogits + r * cols;
    const bool ignored = labels && label < 0;
    for (int64_t c = threadIdx.x; c < cols; c += THREADS) {
      const float p = expf(to_f32(xr[c]) - m) * inv;
      const float t = labels ? (c == label ? 1.f : 0.f) : probs[r * cols + c];
      dr[c] = from_f32<T>(ignored ? 0.f : (p - t) * grad_scale);
    }
  }
}

// Register-resident fused softmax + CE for bf16 rows of up to 512 x 8 x NV
// class-id-targeted columns (the 32000-way vocabulary fits with NV = 8): the
// row is read from memory once into registers (raw bf16, 4 bytes per two
// logits), then max, sum of exponentials and the gradient are computed from
// the registers, recomputing each exponential for the gradient rather than
// keeping 64 floats per thread.  That keeps the kernel at two 512-thread
// blocks per SM, so one block's loads overlap the other's reductions.
// dlogits may alias x: every thread writes only vectors it has already
// loaded, and only after the block-wide reductions.
template <int NV>
__global__ void __launch_bounds__(512, 2) softmax_ce_reg_kernel(const __nv_bfloat16* x, const int* __restrict__ labels,
                                                                float* __restrict__ loss_rows,
                                                                __nv_bfloat16* dlogits, int64_t cols,
                                                                float grad_scale) {
  constexpr int THREADS = 512;
  pdl_wait();
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* xr = x + r * cols;
  const int nvec = (int)(cols / 8);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  uint4 raw[NV];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * THREADS;
    if (v < nvec) raw[i] = reinterpret_cast<const uint4*>(xr)[v];
  }
  const int label = labels[r];
  const float xl = (label >= 0 && label < cols) ? __bfloat162float(xr[label]) : 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * THREADS;
    if (v < nvec) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        mx = fmaxf(mx, fmaxf(f.x, f.y));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[wid] = mx;
  __syncthreads();
  mx = lane < THREADS / 32 ? red[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * THREADS;
    if (v < nvec) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        sum += __expf(f.x - mx) + __expf(f.y - mx);
      }
    }
  }
  sum = warp_sum(sum);
  __syncthreads();  // every warp has read red[] (the maximum)
  if (lane == 0) red[wid] = sum;
  __syncthreads();
  sum = lane < THREADS / 32 ? red[lane] : 0.f;
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  if (threadIdx.x == 0 && loss_rows) loss_rows[r] = label < 0 ? 0.f : mx + logf(sum) - xl;
  const float gs = label < 0 ? 0.f : grad_scale;
  __nv_bfloat16* dr = dlogits + r * cols;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int v = threadIdx.x + i * THREADS;
    if (v >= nvec) continue;
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = v * 8 + 2 * k;
      const float2 f = __bfloat1622float2(h[k]);
      const float g0 = (__expf(f.x - mx) * inv - (c == label ? 1.f : 0.f)) * gs;
      const float g1 = (__expf(f.y - mx) * inv - (c + 1 == label ? 1.f : 0.f)) * gs;
      oh[k] = __floats2bfloat162_rn(g0, g1);
    }
    reinterpret_cast<uint4*>(dr)[v] = o;
  }
}

constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the hardware approximation (ex2.approx.ftz).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// A bf16 pair (first element in the low half) as two floats: a bf16 is the
// upper half of the fp32 of the same value.
__device__ __forceinline__ float2 bf2_unpack(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Persistent form of softmax_ce_reg_kernel: each block walks the rows
// blockIdx.x, + gridDim.x, ... and streams its next row into shared memory
// with cp.async while it reduces the current one from registers, so the
// memory system stays busy through the reductions and the gradient stores
// (two blocks per SM, one 64 KB row buffer each at 32000 columns).  Unlike
// softmax_ce_reg_kernel it computes each exponential once: the sum pass keeps
// exp(x - max) in registers as bf16 in place of the logit, and the gradient
// pass scales it (the label's gradient p - 1 stays in fp32 throughout).
// dlogits may alias x (a row is overwritten only after it has been read, and
// the prefetched row is a different one).
template <int NV>
__global__ void __launch_bounds__(512, 2) softmax_ce_pipe_kernel(const __nv_bfloat16* x, const int* __restrict__ labels,
                                                                 float* __restrict__ loss_rows,
                                                                 __nv_bfloat16* dlogits, int64_t rows, int64_t cols,
                                                                 float grad_scale) {
  constexpr int THREADS = 512;
  pdl_wait();
  extern __shared__ uint4 srow[];
  __shared__ float red[32];
  const int nvec = (int)(cols / 8);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  auto prefetch = [&](int64_t row) {
    if (row < rows) {
      const uint4* src = reinterpret_cast<const uint4*>(x + row * cols);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int v = threadIdx.x + i * THREADS;
        if (v < nvec) sm100::cp_async_16(sm100::smem_u32(srow + v), src + v, 16);
      }
    }
    sm100::cp_async_commit();
  };
  int64_t r = blockIdx.x;
  prefetch(r);
  for (; r < rows; r += gridDim.x) {
    sm100::cp_async_wait<0>();
    __syncthreads();  // the row is in shared memory
    uint4 raw[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * THREADS;
      if (v < nvec) raw[i] = srow[v];
    }
    const int label = labels[r];
    const float xl =
        (label >= 0 && label < cols) ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(srow)[label]) : 0.f;
    __syncthreads();  // every thread has read the buffer
    prefetch(r + gridDim.x);
    // The row maximum on bf16 pairs (exact: a maximum needs no rounding).
    __nv_bfloat162 m2 = __halves2bfloat162(__ushort_as_bfloat16(0xff80), __ushort_as_bfloat16(0xff80));
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * THREADS;
      if (v < nvec) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
        m2 = __hmax2(m2, __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3])));
      }
    }
    float mx = fmaxf(__low2float(m2), __high2float(m2));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[wid] = mx;
    __syncthreads();
    mx = lane < THREADS / 32 ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // The exponentials replace the logits in registers (as bf16), so the
    // gradient pass needs none: non-label gradients carry one extra bf16
    // rounding of p, the same size as the rounding of the stored gradient.
    // exp(x - max) = 2^((x - max) log2(e)), packed in pairs.  The difference
    // comes first: it is exact near the maximum, where a fused
    // x log2(e) - max log2(e) would leave the rounding error of max log2(e)
    // (about 1e-6 at |max| = 20) in every term, and with it in p - 1 of a
    // confident label.
    const float2 l2e = make_float2(kLog2e, kLog2e), nm = make_float2(-mx, -mx);
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * THREADS;
      if (v < nvec) {
        uint32_t* w = reinterpret_cast<uint32_t*>(&raw[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 a = __fmul2_rn(__fadd2_rn(bf2_unpack(w[k]), nm), l2e);
          const float2 e = make_float2(ex2_approx(a.x), ex2_approx(a.y));
          s2 = __fadd2_rn(s2, e);
          w[k] = bf2_pack(e.x, e.y);
        }
      }
    }
    float sum = warp_sum(s2.x + s2.y);
    __syncthreads();  // every warp has read red[] (the maximum)
    if (lane == 0) red[wid] = sum;
    __syncthreads();
    sum = lane < THREADS / 32 ? red[lane] : 0.f;
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    if (threadIdx.x == 0 && loss_rows) loss_rows[r] = label < 0 ? 0.f : mx + logf(sum) - xl;
    const float gs = label < 0 ? 0.f : grad_scale;
    const float gl = (__expf(xl - mx) * inv - 1.f) * gs;  // the label's gradient, from fp32 throughout
    const float2 ginv = make_float2(inv * gs, inv * gs);
    __nv_bfloat16* dr = dlogits + r * cols;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int v = threadIdx.x + i * THREADS;
      if (v >= nvec) continue;
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw[i]);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 g = __fmul2_rn(bf2_unpack(w[k]), ginv);
        ow[k] = bf2_pack(g.x, g.y);
      }
      reinterpret_cast<uint4*>(dr)[v] = o;
    }
    // The label's gradient replaces its p * scale, written by the thread that
    // stored the label's vector (a later store of the same thread).
    if (label >= 0 && label < cols && (label / 8) % THREADS == (int)threadIdx.x) dr[label] = __float2bfloat16_rn(gl);
  }
  sm100::cp_async_wait<0>();
}

// Pointwise losses with a deterministic two-stage sum:
//  MSE:  l = (p - t)^2,                      g = 2 (p - t) * gscale
//  BCE:  l = -(t log p' + (1-t) log(1-p')),  p' = clamp(p, eps, 1-eps),
//        g = (p' - t) / (p' (1 - p')) * gscale
template <typename T>
__global__ void pointwise_loss_kernel(int kind, const T* __restrict__ p, const float* __restrict__ t, int64_t n,
                                      float gscale, T* __restrict__ grad, float* __restrict__ partial) {
  __shared__ float sm[32];
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float pv = to_f32(p[i]), tv = t[i];
    float l, g;
    if (kind == LOSS_MSE) {
      const float d = pv - tv;
      l = d * d;
      g = 2.f * d * gscale;
    } else {
      const float eps = 1e-7f;
      const float pc = fminf(fmaxf(pv, eps), 1.f - eps);
      l = -(tv * logf(pc) + (1.f - tv) * logf(1.f - pc));
      g = (pc - tv) / (pc * (1.f - pc)) * gscale;
    }
    acc += l;
    if (grad) grad[i] = from_f32<T>(g);
  }
  acc = block_sum(acc, sm);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

__global__ void sum_partials_kernel(const float* __restrict__ part, int n, float scale, float* __restrict__ out) {
  __shared__ float sm[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += part[i];
  acc = block_sum(acc, sm);
  if (threadIdx.x == 0) out[0] = acc * scale;
}

// ---- warp-per-row kernels for rows that fit in registers --------------------
// Each lane holds NV 16-byte vectors (EPV elements each) of the row; lane l
// owns vectors l, l+32, ...  Requires cols == 32 * NV * EPV.
template <typename T> struct V16 { static constexpr int EPV = 16 / sizeof(T); };

template <typename T, int NV>
__device__ __forceinline__ void row_load(const T* __restrict__ src, int lane, float (&v)[NV][16 / sizeof(T)]) {
  constexpr int EPV = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const uint4 u = reinterpret_cast<const uint4*>(src)[lane + 32 * i];
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < EPV; ++k) v[i][k] = to_f32(e[k]);
  }
}
template <typename T, int NV>
__device__ __forceinline__ void row_store(T* __restrict__ dst, int lane, const float (&v)[NV][16 / sizeof(T)]) {
  constexpr int EPV = 16 / sizeof(T);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int k = 0; k < EPV; ++k) e[k] = from_f32<T>(v[i][k]);
    reinterpret_cast<uint4*>(dst)[lane + 32 * i] = u;
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                                           int cols, bool log_out) {
  constexpr int EPV = 16 / sizeof(T);
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float v[NV][EPV];
  row_load<T, NV>(x + r * cols, lane, v);
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) m = fmaxf(m, v[i][k]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) {
      const float e = expf(v[i][k] - m);
      s += e;
      if (!log_out) v[i][k] = e;
    }
  s = warp_sum(s);
  if (log_out) {
    const float lse = m + logf(s);
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int k = 0; k < EPV; ++k) v[i][k] -= lse;
  } else {
    const float inv = 1.f / s;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int k = 0; k < EPV; ++k) v[i][k] *= inv;
  }
  row_store<T, NV>(y + r * cols, lane, v);
}

template <typename T, int NV>
__global__ void __launch_bounds__(256) softmax_bwd_warp_kernel(const T* __restrict__ y, const T* __restrict__ dy,
                                                               T* __restrict__ dx, int64_t rows, int cols) {
  constexpr int EPV = 16 / sizeof(T);
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float a[NV][EPV], g[NV][EPV];
  row_load<T, NV>(y + r * cols, lane, a);
  row_load<T, NV>(dy + r * cols, lane, g);
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) dot += a[i][k] * g[i][k];
  dot = warp_sum(dot);
#pragma unroll
  for (int i = 0; i < NV; ++i)
#pragma unroll
    for (int k = 0; k < EPV; ++k) g[i][k] = a[i][k] * (g[i][k] - dot);
  row_store<T, NV>(dx + r * cols, lane, g);
}

// Dispatch to the warp kernels when cols == 32 * NV * EPV for NV in {1,2,4,8}
// and the pointers are 16-byte aligned; returns false otherwise.
template <typename T>
bool try_softmax_warp(const void* x, void* y, int64_t rows, int64_t cols, bool log_out, cudaStream_t s) {
  constexpr int EPV = 16 / sizeof(T);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) return false;
  const unsigned g = (unsigned)((rows + 7) / 8);
  switch (cols / (32 * EPV) * ((cols % (32 * EPV)) == 0)) {
    case 1: softmax_warp_kernel<T, 1><<<g, 256, 0, s>>>((const T*)x, (T*)y, rows, (int)cols, log_out); return true;
    case 2: softmax_warp_kernel<T, 2><<<g, 256, 0, s>>>((const T*)x, (T*)y, rows, (int)cols, log_out); return true;
    case 4: softmax_warp_kernel<T, 4><<<g, 256, 0, s>>>((const T*)x, (T*)y, rows, (int)cols, log_out); return true;
    case 8: softmax_warp_kernel<T, 8><<<g, 256, 0, s>>>((const T*)x, (T*)y, rows, (int)cols, log_out); return true;
    default: return false;
  }
}
template <typename T>
bool try_softmax_bwd_warp(const void* y, const void* dy, void* dx, int64_t rows, int64_t cols, cudaStream_t s) {
  constexpr int EPV = 16 / sizeof(T);
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(dx)) & 15)
    return false;
  const unsigned g = (unsigned)((rows + 7) / 8);
  switch (cols / (32 * EPV) * ((cols % (32 * EPV)) == 0)) {
    case 1: softmax_bwd_warp_kernel<T, 1><<<g, 256, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, rows, (int)cols); return true;
    case 2: softmax_bwd_warp_kernel<T, 2><<<g, 256, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, rows, (int)cols); return true;
    case 4: softmax_bwd_warp_kernel<T, 4><<<g, 256, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, rows, (int)cols); return true;
    case 8: softmax_bwd_warp_kernel<T, 8><<<g, 256, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, rows, (int)cols); return true;
    default: return false;
  }
}

template <typename T>
void launch_softmax(const void* x, void* y, int64_t rows, int64_t cols, bool log_out, cudaStream_t s) {
  if (try_softmax_warp<T>(x, y, rows, cols, log_out, s)) return;
  if (cols <= 64)
    softmax_rows_kernel<T, 32><<<(unsigned)rows, 32, 0, s>>>((const T*)x, (T*)y, cols, log_out);
  else if (cols <= 4096)
    softmax_rows_kernel<T, 128><<<(unsigned)rows, 128, 0, s>>>((const T*)x, (T*)y, cols, log_out);
  else
    softmax_rows_kernel<T, 512><<<(unsigned)rows, 512, 0, s>>>((const T*)x, (T*)y, cols, log_out);
}

template <typename T>
void launch_softmax_bwd(const void* y, const void* dy, void* dx, int64_t rows, int64_t cols, cudaStream_t s) {
  if (try_softmax_bwd_warp<T>(y, dy, dx, rows, cols, s)) return;
  if (cols <= 64)
    softmax_bwd_kernel<T, 32><<<(unsigned)rows, 32, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, cols);
  else
    softmax_bwd_kernel<T, 256><<<(unsigned)rows, 256, 0, s>>>((const T*)y, (const T*)dy, (T*)dx, cols);
}

template <typename T>
void launch_ce(const void* x, const int* labels, const float* probs, float* loss_rows, void* dlogits, int64_t rows,
               int64_t cols, float grad_scale, cudaStream_t s) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dlogits)) & 15) == 0;
    if (labels && dlogits && aligned && cols % 8 == 0 && cols > 4096 && cols <= 512 * 8 * 8) {
      const int64_t per = (cols / 8 + 511) / 512;  // 16-byte vectors per thread
      const auto* xb = (const __nv_bfloat16*)x;
      auto* db = (__nv_bfloat16*)dlogits;
      static const bool pipe = [] {
        const char* e = std::getenv("DLVK_CE_PIPE");
        return !(e && e[0] == '0');
      }();
      const int smem = (int)(cols * 2);
      if (pipe && smem <= 100 * 1024) {
        auto kern = per <= 2 ? softmax_ce_pipe_kernel<2>
                             : (per <= 4 ? softmax_ce_pipe_kernel<4> : softmax_ce_pipe_kernel<8>);
        int sms = 0;
        const int dev = current_device_slot();
        static bool attr[kMaxDevices][3] = {};  // per device and instantiation (set to the largest row size allowed)
        const int ai = per <= 2 ? 0 : (per <= 4 ? 1 : 2);
        if (!attr[dev][ai]) {
          DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
          attr[dev][ai] = true;
        }
        DLVK_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const unsigned grid = (unsigned)std::min<int64_t>(rows, 2 * (int64_t)sms);
        launch_pdl(kern, dim3(grid), dim3(512), smem, s, xb, labels, loss_rows, db, rows, cols, grad_scale);
        return;
      }
      auto kern = per <= 2 ? softmax_ce_reg_kernel<2> : (per <= 4 ? softmax_ce_reg_kernel<4> : softmax_ce_reg_kernel<8>);
      launch_pdl(kern, dim3((unsigned)rows), dim3(512), 0, s, xb, labels, loss_rows, db, cols, grad_scale);
      return;
    }
  }
  if (cols <= 64)
    softmax_ce_kernel<T, 32><<<(unsigned)rows, 32, 0, s>>>((const T*)x, labels, probs, loss_rows, (T*)dlogits, cols,
                                                           grad_scale);
  else if (cols <= 4096)
    softmax_ce_kernel<T, 128><<<(unsigned)rows, 128, 0, s>>>((const T*)x, labels, probs, loss_rows, (T*)dlogits,
                                                             cols, grad_scale);
  else
    softmax_ce_kernel<T, 512><<<(unsigned)rows, 512, 0, s>>>((const T*)x, labels, probs, loss_rows, (T*)dlogits,
                                                             cols, grad_scale);
}

}  // namespace

void softmax(DType dt, const void* x, void* y, int64_t rows, int64_t cols, bool log_out, cudaStream_t s) {
  if (rows == 0) return;
  if (dt == DType::F32) launch_softmax<float>(x, y, rows, cols, log_out, s);
  else if (dt == DType::BF16) launch_softmax<__nv_bfloat16>(x, y, rows, cols, log_out, s);
  else throw std::runtime_error("dlvk::softmax: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void softmax_bwd(DType dt, const void* y, const void* dy, void* dx, int64_t rows, int64_t cols, cudaStream_t s) {
  if (rows == 0) return;
  if (dt == DType::F32) launch_softmax_bwd<float>(y, dy, dx, rows, cols, s);
  else if (dt == DType::BF16) launch_softmax_bwd<__nv_bfloat16>(y, dy, dx, rows, cols, s);
  else throw std::runtime_error("dlvk::softmax_bwd: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void softmax_cross_entropy(DType dt, const void* logits, const int* labels, const float* probs, float* loss_rows,
                           void* dlogits, int64_t rows, int64_t cols, float grad_scale, cudaStream_t s) {
  if (rows == 0) return;
  if (dt == DType::F32) launch_ce<float>(logits, labels, probs, loss_rows, dlogits, rows, cols, grad_scale, s);
  else if (dt == DType::BF16)
    launch_ce<__nv_bfloat16>(logits, labels, probs, loss_rows, dlogits, rows, cols, grad_scale, s);
  else throw std::runtime_error("dlvk::softmax_cross_entropy: unsupported dtype");
  DLVK_POST_LAUNCH();
}

int pointwise_loss_blocks(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>(296, (n + 1023) / 1024)); }

void pointwise_loss(DType dt, int kind, const void* p, const float* t, int64_t n, float loss_scale, float grad_scale,
                    void* grad, float* out, float* scratch, cudaStream_t s) {
  const int blocks = pointwise_loss_blocks(n);
  if (dt == DType::F32)
    pointwise_loss_kernel<float><<<blocks, 256, 0, s>>>(kind, (const float*)p, t, n, grad_scale, (float*)grad, scratch);
  else if (dt == DType::BF16)
    pointwise_loss_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(kind, (const __nv_bfloat16*)p, t, n, grad_scale,
                                                                (__nv_bfloat16*)grad, scratch);
  else throw std::runtime_error("dlvk::pointwise_loss: unsupported dtype");
  DLVK_POST_LAUNCH();
  sum_partials_kernel<<<1, 512, 0, s>>>(scratch, blocks, loss_scale, out);
  DLVK_POST_LAUNCH();
}

void sum_rows_to_scalar(const float* rows_vals, int64_t n, float scale, float* out, cudaStream_t s) {
  sum_partials_kernel<<<1, 1024, 0, s>>>(rows_vals, (int)n, scale, out);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
