// 2-D convolution (NCHW, weight [Cout, Cin, KH, KW]) forward, input-gradient
// and weight/bias-gradient kernels, and max/avg pooling forward/backward.
//
// Reference shaders: conv2d.comp:37-84, conv2d_backward_input.comp:37-89,
// conv2d_backward_weight.comp:37-102, maxpool2d.comp:32-78,
// maxpool2d_backward.comp:27-61, avgpool2d.comp:28-70,
// avgpool2d_backward.comp:28-81 (host dispatch src/tensor/tensor_ops.cpp:
// 1733-1887; the backward dispatchers there are stubs, :1983-2034).
//
// The convolutions of the small-CNN workload have K = Cin*KH*KW of 9 and 72
// and 8/16 output channels: far below one tensor-core tile (K granularity 16,
// N >= 8, and >90% of an M=128 x N=256 tile idle), so they are bandwidth
// bound.  These kernels keep the whole filter bank in shared memory, read
// each input element once per output-channel tile and fuse bias + ReLU (and,
// for the weight gradient, the bias gradient), writing every output once.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

constexpr int kCoTile = 16;

// One thread = one output pixel x kCoTile output channels.
template <typename T>
__global__ void __launch_bounds__(256) conv_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                       const float* __restrict__ bias, T* __restrict__ y, ConvDesc d,
                                                       int relu) {
  extern __shared__ float sw[];  // [kCoTile][Cin*KH*KW]
  const int n = blockIdx.y, co0 = blockIdx.z * kCoTile;
  const int Kel = d.Cin * d.KH * d.KW;
  const int nco = min(kCoTile, d.Cout - co0);
  for (int i = threadIdx.x; i < nco * Kel; i += blockDim.x) sw[i] = to_f32(w[(int64_t)co0 * Kel + i]);
  __syncthreads();
  const int HWo = d.Ho * d.Wo;
  const int pix = blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= HWo) return;
  const int oh = pix / d.Wo, ow = pix - oh * d.Wo;
  float acc[kCoTile];
#pragma unroll
  for (int c = 0; c < kCoTile; ++c) acc[c] = (c < nco && bias) ? bias[co0 + c] : 0.f;
  const T* xn = x + (int64_t)n * d.Cin * d.H * d.W;
  for (int ci = 0; ci < d.Cin; ++ci) {
    for (int kh = 0; kh < d.KH; ++kh) {
      const int ih = oh * d.stride - d.pad + kh;
      if (ih < 0 || ih >= d.H) continue;
      for (int kw = 0; kw < d.KW; ++kw) {
        const int iw = ow * d.stride - d.pad + kw;
        if (iw < 0 || iw >= d.W) continue;
        const float xv = to_f32(xn[((int64_t)ci * d.H + ih) * d.W + iw]);
        const int wi = (ci * d.KH + kh) * d.KW + kw;
#pragma unroll
        for (int c = 0; c < kCoTile; ++c) acc[c] = fmaf(xv, sw[c * Kel + wi], acc[c]);
      }
    }
  }
  T* yn = y + ((int64_t)n * d.Cout + co0) * HWo + pix;
#pragma unroll
  for (int c = 0; c < kCoTile; ++c) {
    if (c < nco) {
      float v = acc[c];
      if (relu) v = fmaxf(v, 0.f);
      yn[(int64_t)c * HWo] = from_f32<T>(v);
    }
  }
}

// dX[n, ci, ih, iw] = sum_{co,kh,kw} g[n, co, oh, ow] * w[co, ci, kh, kw] with
// oh = (ih + pad - kh) / stride when divisible.  Optionally masks by the
// previous layer's ReLU (mask_src > 0), fusing that activation's backward.
template <typename T>
__global__ void __launch_bounds__(256) conv_dgrad_kernel(const T* __restrict__ g, const T* __restrict__ w,
                                                         T* __restrict__ dx, const T* __restrict__ relu_src,
                                                         ConvDesc d) {
  extern __shared__ float sw[];  // full filter bank [Cout][Cin*KH*KW]
  const int Kel = d.Cin * d.KH * d.KW;
  for (int i = threadIdx.x; i < d.Cout * Kel; i += blockDim.x) sw[i] = to_f32(w[i]);
  __syncthreads();
  const int n = blockIdx.y;
  const int HW = d.H * d.W;
  const int64_t tot = (int64_t)d.Cin * HW;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= tot) return;
  const int ci = (int)(e / HW);
  const int rem = (int)(e - (int64_t)ci * HW);
  const int ih = rem / d.W, iw = rem - ih * d.W;
  const int HWo = d.Ho * d.Wo;
  const T* gn = g + (int64_t)n * d.Cout * HWo;
  float acc = 0.f;
  for (int kh = 0; kh < d.KH; ++kh) {
    const int th = ih + d.pad - kh;
    if (th < 0 || th % d.stride) continue;
    const int oh = th / d.stride;
    if (oh >= d.Ho) continue;
    for (int kw = 0; kw < d.KW; ++kw) {
      const int tw = iw + d.pad - kw;
      if (tw < 0 || tw % d.stride) continue;
      const int ow = tw / d.stride;
      if (ow >= d.Wo) continue;
      const int wi = (ci * d.KH + kh) * d.KW + kw;
      for (int co = 0; co < d.Cout; ++co) acc = fmaf(to_f32(gn[(int64_t)co * HWo + oh * d.Wo + ow]), sw[co * Kel + wi], acc);
    }
  }
  const int64_t xi = (int64_t)n * tot + e;
  if (relu_src && !(to_f32(relu_src[xi]) > 0.f)) acc = 0.f;
  dx[xi] = from_f32<T>(acc);
}

// Input gradient with the output gradient staged: one block per chunk of
// images; each image's [Cout][Ho][Wo] gradient and the filter bank sit in
// shared memory (fp32) and each thread computes input elements
// threadIdx.x, + 256, ... of the image (all output channels and taps from
// shared memory, so a warp reads one filter value per step and consecutive
// gradient values).
template <typename T>
__global__ void __launch_bounds__(256) conv_dgrad_image_kernel(const T* __restrict__ g, const T* __restrict__ w,
                                                               T* __restrict__ dx, const T* __restrict__ relu_src,
                                                               ConvDesc d, int ipb) {
  extern __shared__ float dsm[];
  const int Kel = d.Cin * d.KH * d.KW;
  const int HW = d.H * d.W, HWo = d.Ho * d.Wo;
  float* sw = dsm;                  // [Cout][Kel]
  float* sg = dsm + d.Cout * Kel;   // [Cout][Ho][Wo]
  for (int i = threadIdx.x; i < d.Cout * Kel; i += blockDim.x) sw[i] = to_f32(w[i]);
  const int n0 = blockIdx.x * ipb, n1 = min(d.N, n0 + ipb);
  const int tot = d.Cin * HW;
  for (int n = n0; n < n1; ++n) {
    __syncthreads();  // the previous image's gradient is no longer read (and sw is written)
    const T* gn = g + (int64_t)n * d.Cout * HWo;
#pragma unroll 8
    for (int i = threadIdx.x; i < d.Cout * HWo; i += blockDim.x) sg[i] = to_f32(gn[i]);
    __syncthreads();
    for (int e = threadIdx.x; e < tot; e += blockDim.x) {
      const int ci = e / HW;
      const int rem = e - ci * HW;
      const int ih = rem / d.W, iw = rem - ih * d.W;
      float acc = 0.f;
      for (int kh = 0; kh < d.KH; ++kh) {
        const int th = ih + d.pad - kh;
        if (th < 0 || th % d.stride) continue;
        const int oh = th / d.stride;
        if (oh >= d.Ho) continue;
        for (int kw = 0; kw < d.KW; ++kw) {
          const int tw = iw + d.pad - kw;
          if (tw < 0 || tw % d.stride) continue;
          const int ow = tw / d.stride;
          if (ow >= d.Wo) continue;
          const float* gp = sg + oh * d.Wo + ow;
          const float* wp = sw + (ci * d.KH + kh) * d.KW + kw;
#pragma unroll 4
          for (int co = 0; co < d.Cout; ++co) acc = fmaf(gp[co * HWo], wp[co * Kel], acc);
        }
      }
      const int64_t xi = (int64_t)n * tot + e;
      if (relu_src && !(to_f32(relu_src[xi]) > 0.f)) acc = 0.f;
      dx[xi] = from_f32<T>(acc);
    }
  }
}

// Shared memory of conv_dgrad_image_kernel, or 0 when it does not apply.
size_t conv_dgrad_image_smem(const ConvDesc& d) {
  const size_t floats = (size_t)d.Cout * d.Cin * d.KH * d.KW + (size_t)d.Cout * d.Ho * d.Wo;
  const size_t bytes = floats * sizeof(float);
  return (d.Cin * d.H * d.W <= 16384 && bytes <= 96 * 1024) ? bytes : 0;
}

// Weight/bias gradient partials: block (co, chunk) sums over the images of its
// chunk and all output pixels; each thread keeps 32 weight partials in
// registers (weights processed in groups of 32).  The group's input offsets
// (ci, kh, kw) are decoded once (through shared memory into registers), so
// the pixel loop does one bounds test, one load and one fma per weight.  partial[chunk][co][Kel+1]
// (last slot = bias gradient).  Fixed reduction order => deterministic.
template <typename T>
__global__ void __launch_bounds__(256) conv_wgrad_partial_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                                                 float* __restrict__ partial, ConvDesc d,
                                                                 int imgs_per_chunk) {
  __shared__ float red[8][33];
  __shared__ int s_off[32], s_kh[32], s_kw[32];
  const int co = blockIdx.x, chunk = blockIdx.y;
  const int Kel = d.Cin * d.KH * d.KW;
  const int HWo = d.Ho * d.Wo;
  const int64_t HW = (int64_t)d.H * d.W;
  const int n0 = chunk * imgs_per_chunk, n1 = min(d.N, n0 + imgs_per_chunk);
  const int64_t work = (int64_t)(n1 - n0) * HWo;
  float* out = partial + ((int64_t)chunk * d.Cout + co) * (Kel + 1);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int wg = 0; wg < Kel; wg += 32) {
    __syncthreads();  // the previous group's tables and red[] are no longer read
    if (threadIdx.x < 32) {
      const int wi = wg + threadIdx.x;
      if (wi < Kel) {
        const int ci = wi / (d.KH * d.KW);
        const int r = wi - ci * d.KH * d.KW;
        const int kh = r / d.KW, kw = r - kh * d.KW;
        s_off[threadIdx.x] = (int)(ci * HW) + kh * d.W + kw;
        s_kh[threadIdx.x] = kh;
        s_kw[threadIdx.x] = kw;
      } else {  // past the last weight: never in range
        s_off[threadIdx.x] = 0;
        s_kh[threadIdx.x] = -(1 << 14);
        s_kw[threadIdx.x] = 0;
      }
    }
    __syncthreads();
    float acc[32];
    int toff[32], tkw[32];  // the table in registers: input offset, and kh << 16 | kw
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      acc[j] = 0.f;
      toff[j] = s_off[j];
      tkw[j] = (s_kh[j] << 16) | (s_kw[j] & 0xffff);
    }
    float bacc = 0.f;
    for (int64_t it = threadIdx.x; it < work; it += blockDim.x) {
      const int n = n0 + (int)(it / HWo);
      const int pix = (int)(it - (int64_t)(n - n0) * HWo);
      const int oh = pix / d.Wo, ow = pix - oh * d.Wo;
      const float gv = to_f32(g[((int64_t)n * d.Cout + co) * HWo + pix]);
      if (gv == 0.f) continue;
      bacc += gv;
      const int ih0 = oh * d.stride - d.pad, iw0 = ow * d.stride - d.pad;
      const int64_t base = ((int64_t)n * d.Cin * d.H + ih0) * d.W + iw0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int ih = ih0 + (tkw[j] >> 16), iw = iw0 + (short)(tkw[j] & 0xffff);
        if ((unsigned)ih < (unsigned)d.H && (unsigned)iw < (unsigned)d.W)
          acc[j] = fmaf(gv, to_f32(x[base + toff[j]]), acc[j]);
      }
    }
    // Block reduction of the 32 partials (and, in the first group, the bias
    // sum): warp shuffle then across warps.
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float v = warp_sum(acc[j]);
      if (lane == j) red[wid][j] = v;
    }
    if (wg == 0) {
      const float v = warp_sum(bacc);
      if (lane == 0) red[wid][32] = v;
    }
    __syncthreads();
    if (threadIdx.x < 33) {
      float sum = 0.f;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) sum += red[i][threadIdx.x];
      if (threadIdx.x < 32) {
        if (wg + (int)threadIdx.x < Kel) out[wg + threadIdx.x] = sum;
      } else if (wg == 0) {
        out[Kel] = sum;
      }
    }
  }
}

// Sum the chunk partials: dw[co, wi] (+)= sum_chunk partial[chunk][co][wi].
// Weight gradient of a 3 x 3 convolution with few channels, one block per
// chunk of images: each image's input planes and output gradient are staged
// in shared memory (fp32), and thread t owns the (co, ci) channel pair
// t % (Cout * Cin) over pixel group t / (Cout * Cin): it reads the gradient
// once per pixel and accumulates all nine taps of that pair (and, for ci = 0,
// the bias sum).  Groups are combined in shared memory in a fixed order; the
// block writes its partial in conv_wgrad_partial_kernel's layout
// [chunk][Cout][Cin * 9 + 1], so conv_wgrad_final_kernel finishes both.
template <typename T>
__global__ void __launch_bounds__(256) conv_wgrad_image_kernel(const T* __restrict__ x, const T* __restrict__ g,
                                                               float* __restrict__ partial, ConvDesc d, int ipb) {
  extern __shared__ float wsm[];
  const int HW = d.H * d.W, HWo = d.Ho * d.Wo;
  const int pairs = d.Cout * d.Cin;
  const int G = max(1, (int)blockDim.x / pairs);  // pixel groups
  const int Kel = d.Cin * 9;
  float* sx = wsm;                       // [Cin][H][W]
  float* sg = sx + d.Cin * HW;           // [Cout][Ho][Wo]
  float* sred = sg + d.Cout * HWo;       // [G][pairs][10] group partials
  const int n0 = blockIdx.x * ipb, n1 = min(d.N, n0 + ipb);
  const int grp = threadIdx.x / pairs;
  const int pr = threadIdx.x - grp * pairs;
  const bool active = grp < G && pr < pairs;
  const int co = active ? pr / d.Cin : 0, ci = active ? pr - co * d.Cin : 0;
  float acc[10];
#pragma unroll
  for (int k = 0; k < 10; ++k) acc[k] = 0.f;
  for (int n = n0; n < n1; ++n) {
    __syncthreads();  // the previous image's planes are no longer read
    const T* xn = x + (int64_t)n * d.Cin * HW;
    const T* gn = g + (int64_t)n * d.Cout * HWo;
    // unrolled so that several loads per thread are in flight
#pragma unroll 8
    for (int i = threadIdx.x; i < d.Cin * HW; i += blockDim.x) sx[i] = to_f32(xn[i]);
#pragma unroll 8
    for (int i = threadIdx.x; i < d.Cout * HWo; i += blockDim.x) sg[i] = to_f32(gn[i]);
    __syncthreads();
    if (!active) continue;
    const float* gp = sg + co * HWo;
    const float* xp = sx + ci * HW;
    int oh = grp / d.Wo, ow = grp - oh * d.Wo;
    for (int pix = grp; pix < HWo; pix += G) {
      const float gv = gp[pix];
      acc[9] += gv;
      const int ih0 = oh * d.stride - d.pad, iw0 = ow * d.stride - d.pad;
#pragma unroll
      for (int kh = 0; kh < 3; ++kh) {
        const int ih = ih0 + kh;
        if ((unsigned)ih >= (unsigned)d.H) continue;
#pragma unroll
        for (int kw = 0; kw < 3; ++kw) {
          const int iw = iw0 + kw;
          if ((unsigned)iw < (unsigned)d.W) acc[kh * 3 + kw] = fmaf(gv, xp[ih * d.W + iw], acc[kh * 3 + kw]);
        }
      }
      ow += G;
      while (ow >= d.Wo) {
        ow -= d.Wo;
        ++oh;
      }
    }
  }
  __syncthreads();
  if (active) {
#pragma unroll
    for (int k = 0; k < 10; ++k) sred[((int64_t)grp * pairs + pr) * 10 + k] = acc[k];
  }
  __syncthreads();
  float* out = partial + (int64_t)blockIdx.x * d.Cout * (Kel + 1);
  for (int i = threadIdx.x; i < pairs * 10; i += blockDim.x) {
    const int q = i / 10, k = i - q * 10;
    float sum = 0.f;
    for (int gg = 0; gg < G; ++gg) sum += sred[((int64_t)gg * pairs + q) * 10 + k];
    const int oc = q / d.Cin, ic = q - oc * d.Cin;
    if (k < 9) out[oc * (Kel + 1) + ic * 9 + k] = sum;
    else if (ic == 0) out[oc * (Kel + 1) + Kel] = sum;  // bias: counted once per output channel
  }
}

// Shared memory of conv_wgrad_image_kernel, or 0 when the shape is not its case.
size_t conv_wgrad_image_smem(const ConvDesc& d) {
  if (d.KH != 3 || d.KW != 3) return 0;
  const int pairs = d.Cout * d.Cin;
  if (pairs > 256) return 0;
  const int G = std::max(1, 256 / pairs);
  const size_t floats = (size_t)d.Cin * d.H * d.W + (size_t)d.Cout * d.Ho * d.Wo + (size_t)G * pairs * 10;
  const size_t bytes = floats * sizeof(float);
  return bytes <= 96 * 1024 ? bytes : 0;
}

// Sums the per-chunk partials: a block covers 32 entries with 8 threads per
// entry, each summing every 8th chunk; the 8 are combined in a fixed order.
__global__ void __launch_bounds__(256) conv_wgrad_final_kernel(const float* __restrict__ partial, int chunks, int Cout,
                                                               int Kel, float* __restrict__ dw,
                                                               float* __restrict__ db, int accumulate) {
  __shared__ float red[8][33];
  const int i = blockIdx.x * 32 + threadIdx.x;
  const int per = Kel + 1;
  float sv = 0.f;
  if (i < Cout * per)
    for (int c = threadIdx.y; c < chunks; c += 8) sv += partial[(int64_t)c * Cout * per + i];
  red[threadIdx.y][threadIdx.x] = sv;
  __syncthreads();
  if (threadIdx.y != 0 || i >= Cout * per) return;
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x];
  const int co = i / per, wi = i - co * per;
  if (wi < Kel) {
    float* p = dw + co * Kel + wi;
    *p = accumulate ? *p + s : s;
  } else if (db) {
    db[co] = accumulate ? db[co] + s : s;
  }
}

// Max pooling, window k x k, stride s, no padding.  idx = flat h*W+w of the
// first maximum in the window (strict '>', src/layers/pooling_layers.cpp:63-99).
template <typename T>
__global__ void maxpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int32_t* __restrict__ idx,
                                   int64_t planes, int H, int W, int Ho, int Wo, int k, int s) {
  const int64_t tot = planes * Ho * Wo;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pl = i / (Ho * Wo);
    const int r = (int)(i - pl * Ho * Wo);
    const int oh = r / Wo, ow = r - oh * Wo;
    const T* xp = x + pl * H * W;
    float best = -INFINITY;
    int bi = (oh * s) * W + ow * s;
    for (int kh = 0; kh < k; ++kh)
      for (int kw = 0; kw < k; ++kw) {
        const int ih = oh * s + kh, iw = ow * s + kw;
        const float v = to_f32(xp[ih * W + iw]);
        if (v > best) {
          best = v;
          bi = ih * W + iw;
        }
      }
    y[i] = from_f32<T>(best);
    if (idx) idx[i] = bi;
  }
}

// Gather form (deterministic, handles overlapping windows): every input pixel
// sums the gradients of the outputs whose argmax it is.
template <typename T>
__global__ void maxpool_bwd_kernel(const T* __restrict__ g, const int32_t* __restrict__ idx, T* __restrict__ dx,
                                   int64_t planes, int H, int W, int Ho, int Wo, int k, int s) {
  const int64_t tot = planes * H * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pl = i / (H * W);
    const int r = (int)(i - pl * H * W);
    const int ih = r / W, iw = r - ih * W;
    const int oh0 = max(0, (ih - k + s) / s), oh1 = min(Ho - 1, ih / s);
    const int ow0 = max(0, (iw - k + s) / s), ow1 = min(Wo - 1, iw / s);
    float acc = 0.f;
    for (int oh = oh0; oh <= oh1; ++oh)
      for (int ow = ow0; ow <= ow1; ++ow) {
        const int64_t o = pl * Ho * Wo + oh * Wo + ow;
        if (idx[o] == r) acc += to_f32(g[o]);
      }
    dx[i] = from_f32<T>(acc);
  }
}

// Average pooling with count_include_pad = false (divide by the number of
// in-bounds taps), forward and backward with the same divisor.
template <typename T>
__global__ void avgpool_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t planes, int H, int W, int Ho,
                                   int Wo, int k, int s, int pad) {
  const int64_t tot = planes * Ho * Wo;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pl = i / (Ho * Wo);
    const int r = (int)(i - pl * Ho * Wo);
    const int oh = r / Wo, ow = r - oh * Wo;
    float acc = 0.f;
    int cnt = 0;
    for (int kh = 0; kh < k; ++kh)
      for (int kw = 0; kw < k; ++kw) {
        const int ih = oh * s - pad + kh, iw = ow * s - pad + kw;
        if (ih < 0 || ih >= H || iw < 0 || iw >= W) continue;
        acc += to_f32(x[pl * H * W + ih * W + iw]);
        ++cnt;
      }
    y[i] = from_f32<T>(cnt ? acc / cnt : 0.f);
  }
}

template <typename T>
__global__ void avgpool_bwd_kernel(const T* __restrict__ g, T* __restrict__ dx, int64_t planes, int H, int W, int Ho,
                                   int Wo, int k, int s, int pad) {
  const int64_t tot = planes * H * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < tot; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pl = i / (H * W);
    const int r = (int)(i - pl * H * W);
    const int ih = r / W, iw = r - ih * W;
    float acc = 0.f;
    for (int kh = 0; kh < k; ++kh) {
      const int th = ih + pad - kh;
      if (th < 0 || th % s) continue;
      const int oh = th / s;
      if (oh >= Ho) continue;
      for (int kw = 0; kw < k; ++kw) {
        const int tw = iw + pad - kw;
        if (tw < 0 || tw % s) continue;
        const int ow = tw / s;
        if (ow >= Wo) continue;
        int cnt = 0;
        for (int a = 0; a < k; ++a)
          for (int b = 0; b < k; ++b) {
            const int h2 = oh * s - pad + a, w2 = ow * s - pad + b;
            if (h2 >= 0 && h2 < H && w2 >= 0 && w2 < W) ++cnt;
          }
        acc += to_f32(g[pl * Ho * Wo + oh * Wo + ow]) / cnt;
      }
    }
    dx[i] = from_f32<T>(acc);
  }
}

inline unsigned grid1d(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace

void conv2d_fwd(DType dt, const void* x, const void* w, const float* bias, void* y, const ConvDesc& d, bool relu,
                cudaStream_t s) {
  const int Kel = d.Cin * d.KH * d.KW;
  const size_t smem = (size_t)kCoTile * Kel * sizeof(float);
  DLVK_CHECK(smem <= 200 * 1024, "conv2d_fwd: filter tile too large for shared memory");
  dim3 grid((unsigned)((d.Ho * d.Wo + 255) / 256), (unsigned)d.N, (unsigned)((d.Cout + kCoTile - 1) / kCoTile));
  if (dt == DType::F32) {
    if (smem > 48 * 1024)
      DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_fwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    conv_fwd_kernel<float><<<grid, 256, smem, s>>>((const float*)x, (const float*)w, bias, (float*)y, d, relu);
  } else if (dt == DType::BF16) {
    if (smem > 48 * 1024)
      DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_fwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
    conv_fwd_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w, bias,
                                                           (__nv_bfloat16*)y, d, relu);
  } else {
    throw std::runtime_error("dlvk::conv2d_fwd: unsupported dtype");
  }
  DLVK_POST_LAUNCH();
}

void conv2d_dgrad(DType dt, const void* g, const void* w, void* dx, const void* relu_src, const ConvDesc& d,
                  cudaStream_t s) {
  const size_t smem = (size_t)d.Cout * d.Cin * d.KH * d.KW * sizeof(float);
  DLVK_CHECK(smem <= 200 * 1024, "conv2d_dgrad: filter bank too large for shared memory");
  const size_t ismem = conv_dgrad_image_smem(d);
  if (ismem > 0 && (dt == DType::F32 || dt == DType::BF16)) {
    const int chunks = std::max(1, std::min(d.N, 1024));
    const int per = (d.N + chunks - 1) / chunks;
    auto launch = [&](auto kern, const auto* gp, const auto* wp, auto* dxp, const auto* rp) {
      if (ismem > 48 * 1024)
        DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ismem));
      kern<<<(unsigned)chunks, 256, ismem, s>>>(gp, wp, dxp, rp, d, per);
    };
    if (dt == DType::F32)
      launch(conv_dgrad_image_kernel<float>, (const float*)g, (const float*)w, (float*)dx, (const float*)relu_src);
    else
      launch(conv_dgrad_image_kernel<__nv_bfloat16>, (const __nv_bfloat16*)g, (const __nv_bfloat16*)w,
             (__nv_bfloat16*)dx, (const __nv_bfloat16*)relu_src);
    DLVK_POST_LAUNCH();
    return;
  }
  const int64_t per_img = (int64_t)d.Cin * d.H * d.W;
  dim3 grid((unsigned)((per_img + 255) / 256), (unsigned)d.N);
  if (dt == DType::F32) {
    if (smem > 48 * 1024)
      DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_dgrad_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    conv_dgrad_kernel<float><<<grid, 256, smem, s>>>((const float*)g, (const float*)w, (float*)dx,
                                                     (const float*)relu_src, d);
  } else if (dt == DType::BF16) {
    if (smem > 48 * 1024)
      DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_dgrad_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    conv_dgrad_kernel<__nv_bfloat16><<<grid, 256, smem, s>>>((const __nv_bfloat16*)g, (const __nv_bfloat16*)w,
                                                             (__nv_bfloat16*)dx, (const __nv_bfloat16*)relu_src, d);
  } else {
    throw std::runtime_error("dlvk::conv2d_dgrad: unsupported dtype");
  }
  DLVK_POST_LAUNCH();
}

// One image per chunk on the staged 3 x 3 path (up to 1024 chunks), 64 chunks otherwise.
int conv2d_wgrad_chunks(const ConvDesc& d) {
  if (conv_wgrad_image_smem(d) > 0) return std::max(1, std::min(d.N, 1024));
  return std::max(1, std::min(d.N, 64));
}
int64_t conv2d_wgrad_scratch_floats(const ConvDesc& d) {
  return (int64_t)conv2d_wgrad_chunks(d) * d.Cout * (d.Cin * d.KH * d.KW + 1);
}

void conv2d_wgrad(DType dt, const void* x, const void* g, float* dw, float* db, bool accumulate, const ConvDesc& d,
                  float* scratch, cudaStream_t s) {
  const int chunks = conv2d_wgrad_chunks(d);
  const int per = (d.N + chunks - 1) / chunks;
  const size_t ismem = conv_wgrad_image_smem(d);
  if (ismem > 0 && (dt == DType::F32 || dt == DType::BF16)) {
    auto launch = [&](auto kern, const auto* xp, const auto* gp) {
      if (ismem > 48 * 1024)
        DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ismem));
      kern<<<(unsigned)chunks, 256, ismem, s>>>(xp, gp, scratch, d, per);
    };
    if (dt == DType::F32)
      launch(conv_wgrad_image_kernel<float>, (const float*)x, (const float*)g);
    else
      launch(conv_wgrad_image_kernel<__nv_bfloat16>, (const __nv_bfloat16*)x, (const __nv_bfloat16*)g);
    DLVK_POST_LAUNCH();
    const int Kel = d.Cin * d.KH * d.KW;
    const int tot = d.Cout * (Kel + 1);
    conv_wgrad_final_kernel<<<(tot + 31) / 32, dim3(32, 8), 0, s>>>(scratch, chunks, d.Cout, Kel, dw, db, accumulate ? 1 : 0);
    DLVK_POST_LAUNCH();
    return;
  }
  dim3 grid((unsigned)d.Cout, (unsigned)chunks);
  if (dt == DType::F32)
    conv_wgrad_partial_kernel<float><<<grid, 256, 0, s>>>((const float*)x, (const float*)g, scratch, d, per);
  else if (dt == DType::BF16)
    conv_wgrad_partial_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)g,
                                                                  scratch, d, per);
  else
    throw std::runtime_error("dlvk::conv2d_wgrad: unsupported dtype");
  DLVK_POST_LAUNCH();
  const int Kel = d.Cin * d.KH * d.KW;
  const int tot = d.Cout * (Kel + 1);
  conv_wgrad_final_kernel<<<(tot + 31) / 32, dim3(32, 8), 0, s>>>(scratch, chunks, d.Cout, Kel, dw, db, accumulate ? 1 : 0);
  DLVK_POST_LAUNCH();
}

void maxpool2d_fwd(DType dt, const void* x, void* y, int32_t* idx, int64_t planes, int H, int W, int k, int stride,
                   cudaStream_t s) {
  const int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
  const unsigned g = grid1d(planes * Ho * Wo);
  if (dt == DType::F32)
    maxpool_fwd_kernel<float><<<g, 256, 0, s>>>((const float*)x, (float*)y, idx, planes, H, W, Ho, Wo, k, stride);
  else if (dt == DType::BF16)
    maxpool_fwd_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, idx, planes, H, W,
                                                        Ho, Wo, k, stride);
  else
    throw std::runtime_error("dlvk::maxpool2d_fwd: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void maxpool2d_bwd(DType dt, const void* g, const int32_t* idx, void* dx, int64_t planes, int H, int W, int k,
                   int stride, cudaStream_t s) {
  const int Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
  const unsigned gr = grid1d(planes * H * W);
  if (dt == DType::F32)
    maxpool_bwd_kernel<float><<<gr, 256, 0, s>>>((const float*)g, idx, (float*)dx, planes, H, W, Ho, Wo, k, stride);
  else if (dt == DType::BF16)
    maxpool_bwd_kernel<__nv_bfloat16><<<gr, 256, 0, s>>>((const __nv_bfloat16*)g, idx, (__nv_bfloat16*)dx, planes, H,
                                                         W, Ho, Wo, k, stride);
  else
    throw std::runtime_error("dlvk::maxpool2d_bwd: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void avgpool2d_fwd(DType dt, const void* x, void* y, int64_t planes, int H, int W, int k, int stride, int pad,
                   cudaStream_t s) {
  const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  const unsigned g = grid1d(planes * Ho * Wo);
  if (dt == DType::F32)
    avgpool_fwd_kernel<float><<<g, 256, 0, s>>>((const float*)x, (float*)y, planes, H, W, Ho, Wo, k, stride, pad);
  else if (dt == DType::BF16)
    avgpool_fwd_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, planes, H, W, Ho,
                                                        Wo, k, stride, pad);
  else
    throw std::runtime_error("dlvk::avgpool2d_fwd: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void avgpool2d_bwd(DType dt, const void* g, void* dx, int64_t planes, int H, int W, int k, int stride, int pad,
                   cudaStream_t s) {
  const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
  const unsigned gr = grid1d(planes * H * W);
  if (dt == DType::F32)
    avgpool_bwd_kernel<float><<<gr, 256, 0, s>>>((const float*)g, (float*)dx, planes, H, W, Ho, Wo, k, stride, pad);
  else if (dt == DType::BF16)
    avgpool_bwd_kernel<__nv_bfloat16><<<gr, 256, 0, s>>>((const __nv_bfloat16*)g, (__nv_bfloat16*)dx, planes, H, W,
                                                         Ho, Wo, k, stride, pad);
  else
    throw std::runtime_error("dlvk::avgpool2d_bwd: unsupported dtype");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
