// Implicit-GEMM convolution on the sm_100a tensor cores (tcgen05 + TMEM).
// Replaces the reference's conv2d shaders (shaders/conv2d_forward.comp,
// conv2d_backward_input.comp, conv2d_backward_weight.comp, dispatched from
// src/tensor/tensor_ops.cpp conv2d paths and src/core/layers.cpp
// Conv2DLayer) for bf16 convolutions whose channel counts are multiples of 8.
//
// The im2col matrix is never materialised.  Activations are gathered in
// NHWC (channels innermost), so every 16-byte vector of a GEMM row is 8
// consecutive channels of one input pixel and one filter tap:
//
//  forward   Y[p, oc]  = sum_k A[p, k] W[oc, k],  k = (kh, kw, c)
//            A[p, k]   = X[n, oh*s - pad + kh, ow*s - pad + kw, c]
//  dgrad     dX[p, c]  = sum_k A[p, k] Wt[c, k],  k = (kh, kw, oc)
//            A[p, k]   = dY[n, (ih + pad - kh)/s, (iw + pad - kw)/s, oc]
//                        (zero unless both divisions are exact)
//  wgrad     dW[oc, k] = sum_p dY[p, oc] A[p, k]  (split over p, fp32 partials)
//
// Kernel layout (persistent, one CTA per SM, 288 threads = 9 warps):
//   warp 0     TMEM allocator + MMA issuer (one lane): 128 x BN x 16 UMMAs
//   warps 1-4  epilogue: tcgen05.ld -> bias / ReLU / ReLU-mask -> global
//   warps 5-8  producers: one thread per 128-byte smem row gathers its eight
//              16-byte vectors with cp.async (zero-fill for padding), fences
//              them into the async proxy and arrives on the stage barrier;
//              thread 0 also loads the dense operand (packed weights for
//              forward/dgrad, dY for wgrad) with a TMA tiled load.
// Every mbarrier wait is bounded and reports through the device error word.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/sm100.h"
#include "dlvk/tmap.h"

namespace dlvk {
namespace {

using namespace sm100;

constexpr int CBM = 128;       // GEMM rows per tile
constexpr int CBK = 64;        // bf16 K elements per 128-byte row
constexpr int KTAB_MAX = 1152; // 8-channel K vectors of one filter (K <= 9216)
constexpr int IG_THREADS = 288;

struct IgemmParams {
  const __nv_bfloat16* src;  // NHWC [Nb, Hs, Ws, Cs]
  int Hs, Ws, Cs;
  int Ho, Wo;                // GEMM rows: P = Nb * Ho * Wo pixels
  int KW, stride, pad;
  int transposed;            // 0: forward gather; 1: dgrad gather
  int P, Ncols, K, num_kb, tiles_m, tiles_n;
  void* out;                 // NCHW [Nb, Ncols, Ho, Wo]
  int out_f32;
  const float* bias;         // [Ncols] or null
  int relu;
  const void* mask;          // NCHW like out (same dtype) or null: out = 0 where mask <= 0
  uint32_t* err;
};

struct WgradParams {
  const __nv_bfloat16* x;    // NHWC forward input [Nb, H, W, C]
  int H, W, C;
  int Ho, Wo, KW, stride, pad;
  int P, OC, Kc, num_kb;     // GEMM: M = OC, N = Kc = KH*KW*C, K = P
  int tiles_m, tiles_n, splits, kb_per_split;
  float* ws;                 // [splits][OC][Kc]
  uint32_t* err;
};

template <int BN>
struct IgCfg {
  static constexpr int A_BYTES = CBM * CBK * 2;
  static constexpr int B_BYTES = BN * CBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 5;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + KTAB_MAX * 8;
};

// K-vector table: entry v describes K elements [8v, 8v+8): channel offset and
// filter tap (kh, kw); c = -1 past the end of K (zero padding).
__device__ __forceinline__ void build_ktab(int2* ktab, int nvec, int K, int Cs, int KW) {
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    const int k = v * 8;
    int2 e = make_int2(-1, 0);
    if (k < K) {
      const int tap = k / Cs;
      const int kh = tap / KW;
      e.x = k - tap * Cs;
      e.y = (kh << 16) | (tap - kh * KW);
    }
    ktab[v] = e;
  }
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int BN>
__global__ void __launch_bounds__(IG_THREADS, 1)
    conv_igemm_kernel(const __grid_constant__ CUtensorMap tmW, IgemmParams p) {
  using C = IgCfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int2* ktab = reinterpret_cast<int2*>(smem + C::STAGES * C::STAGE_BYTES + 256);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;

  build_ktab(ktab, p.num_kb * 8, p.K, p.Cs, p.KW);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 129);  // 128 producer arrivals + the TMA expect_tx arrival
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmW);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 5) {
    // ---- producers: gather A rows, TMA the weight tile ----
    const int g = threadIdx.x - 160;
    const uint32_t swz = (uint32_t)(g & 7);
    const uint32_t row_off = (uint32_t)((g >> 3) * 1024 + (g & 7) * 128);
    const int hw = p.Ho * p.Wo;
    int stage = 0, pend = -1;
    uint32_t phase = 0;
    bool alive = true;
    for (int t = blockIdx.x; t < num_tiles && alive; t += gridDim.x) {
      const int tm = t / p.tiles_n, tn = t - tm * p.tiles_n;
      const int m = tm * CBM + g;
      const bool row_ok = m < p.P;
      int n_img = 0, bh = 0, bw = 0;
      if (row_ok) {
        n_img = m / hw;
        const int r = m - n_img * hw;
        const int oh = r / p.Wo, ow = r - oh * p.Wo;
        bh = p.transposed ? oh + p.pad : oh * p.stride - p.pad;
        bw = p.transposed ? ow + p.pad : ow * p.stride - p.pad;
      }
      const __nv_bfloat16* img = p.src + (int64_t)n_img * p.Hs * p.Ws * p.Cs;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
          alive = false;
          break;
        }
        uint8_t* sA = smem + stage * C::STAGE_BYTES;
        if (g == 0) {
          mbar_arrive_expect_tx(&full[stage], C::B_BYTES);
          tma_load_2d(sA + C::A_BYTES, &tmW, &full[stage], kb * CBK, tn * BN);
        }
        const uint32_t dst = smem_u32(sA) + row_off;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int2 e = ktab[kb * 8 + j];
          const int dh = e.y >> 16, dw = e.y & 0xffff;
          bool ok = row_ok && e.x >= 0;
          int sh, sw;
          if (!p.transposed) {
            sh = bh + dh;
            sw = bw + dw;
          } else if (p.stride == 1) {  // uniform branch: no division on the common path
            sh = bh - dh;
            sw = bw - dw;
          } else {
            const int th = bh - dh, tw = bw - dw;
            ok = ok && th >= 0 && tw >= 0 && (th % p.stride) == 0 && (tw % p.stride) == 0;
            sh = th / p.stride;
            sw = tw / p.stride;
          }
          ok = ok && sh >= 0 && sh < p.Hs && sw >= 0 && sw < p.Ws;
          const __nv_bfloat16* src = ok ? img + ((int64_t)sh * p.Ws + sw) * p.Cs + e.x : p.src;
          cp_async_16(dst + (((uint32_t)j ^ swz) << 4), src, ok ? 16u : 0u);
        }
        cp_async_commit();
        if (pend >= 0) {  // the previous stage's copies are done: publish it
          cp_async_wait<1>();
          fence_proxy_async_smem();
          mbar_arrive(&full[pend]);
        }
        pend = stage;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    cp_async_wait<0>();
    if (pend >= 0 && alive) {
      fence_proxy_async_smem();
      mbar_arrive(&full[pend]);
    }
  } else if (warp == 0) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = make_idesc(1, 1, 1, false, false, CBM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t bBase = aBase + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < CBK / 16; ++k)
            mma_f16(d, make_sw128_desc(aBase + k * 32, 16, 1024), make_sw128_desc(bBase + k * 32, 16, 1024), idesc,
                    (kb != 0 || k != 0) ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 ----
    const int q = warp & 3;
    const int hw = p.Ho * p.Wo;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      const int tm = t / p.tiles_n, tn = t - tm * p.tiles_n;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int m = tm * CBM + q * 32 + lane;
      const bool row_ok = m < p.P;
      const int n_img = row_ok ? m / hw : 0;
      const int64_t obase = (int64_t)n_img * p.Ncols * hw + (m - n_img * hw);
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int i = 0; i < BN / 32; ++i) {
        uint32_t r[32];
        tmem_ld32(tb + (uint32_t)(i * 32), r);
        tmem_ld_wait();
        const int c0 = tn * BN + i * 32;
        if (!row_ok || c0 >= p.Ncols) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        const int nv = min(32, p.Ncols - c0);
        if (p.bias) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) v[j] += p.bias[c0 + j];
        }
        if (p.relu) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
        }
        if (p.mask) {
          if (p.out_f32) {
            const float* mk = reinterpret_cast<const float*>(p.mask) + obase + (int64_t)c0 * hw;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nv && !(mk[(int64_t)j * hw] > 0.f)) v[j] = 0.f;
          } else {
            const __nv_bfloat16* mk = reinterpret_cast<const __nv_bfloat16*>(p.mask) + obase + (int64_t)c0 * hw;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nv && !(__bfloat162float(mk[(int64_t)j * hw]) > 0.f)) v[j] = 0.f;
          }
        }
        if (p.out_f32) {
          float* o = reinterpret_cast<float*>(p.out) + obase + (int64_t)c0 * hw;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) o[(int64_t)j * hw] = v[j];
        } else {
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + obase + (int64_t)c0 * hw;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nv) o[(int64_t)j * hw] = __float2bfloat16_rn(v[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Weight gradient: GEMM rows = output channels (A = dY^T, read M-major from
// NHWC dY by TMA), columns = (kh, kw, c) (B = im2col(X), gathered N-major),
// reduction over pixels split across CTAs into fp32 partials.
constexpr int WG_BN = 128;
struct WgCfg {
  static constexpr int A_BYTES = CBM * CBK * 2;
  static constexpr int B_BYTES = WG_BN * CBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 5;
  static constexpr int TMEM_COLS = 2 * WG_BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + KTAB_MAX * 8;
};

__global__ void __launch_bounds__(IG_THREADS, 1)
    conv_wgrad_kernel(const __grid_constant__ CUtensorMap tmDy, WgradParams p) {
  using C = WgCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int2* ktab = reinterpret_cast<int2*>(smem + C::STAGES * C::STAGE_BYTES + 256);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_split = p.tiles_m * p.tiles_n;
  const int num_units = per_split * p.splits;

  build_ktab(ktab, p.tiles_n * (WG_BN / 8), p.Kc, p.C, p.KW);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 129);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmDy);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto unit_coords = [&](int u, int& tm, int& tn, int& kb0, int& kb1) {
    const int sp = u / per_split;
    const int r = u - sp * per_split;
    tm = r / p.tiles_n;
    tn = r - tm * p.tiles_n;
    kb0 = sp * p.kb_per_split;
    kb1 = min(p.num_kb, kb0 + p.kb_per_split);
  };

  if (warp >= 5) {
    // ---- producers: thread g gathers pixel row (g % 64) of N-chunk g / 64 ----
    const int g = threadIdx.x - 160;
    const int r = g & 63, jn = g >> 6;
    const uint32_t swz = (uint32_t)(r & 7);
    const uint32_t row_off = (uint32_t)(C::A_BYTES + jn * 8192 + (r >> 3) * 1024 + (r & 7) * 128);
    const int hw = p.Ho * p.Wo;
    int stage = 0, pend = -1;
    uint32_t phase = 0;
    bool alive = true;
    for (int u = blockIdx.x; u < num_units && alive; u += gridDim.x) {
      int tm, tn, kb0, kb1;
      unit_coords(u, tm, tn, kb0, kb1);
      const int2* kt = ktab + tn * (WG_BN / 8) + jn * 8;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) {
          alive = false;
          break;
        }
        uint8_t* sA = smem + stage * C::STAGE_BYTES;
        if (g == 0) {
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES);
          tma_load_2d(sA, &tmDy, &full[stage], tm * CBM, kb * CBK);
          tma_load_2d(sA + 8192, &tmDy, &full[stage], tm * CBM + 64, kb * CBK);
        }
        const int m = kb * CBK + r;  // pixel of dY
        const bool row_ok = m < p.P;
        int n_img = 0, bh = 0, bw = 0;
        if (row_ok) {
          n_img = m / hw;
          const int rr = m - n_img * hw;
          const int oh = rr / p.Wo, ow = rr - oh * p.Wo;
          bh = oh * p.stride - p.pad;
          bw = ow * p.stride - p.pad;
        }
        const __nv_bfloat16* img = p.x + (int64_t)n_img * p.H * p.W * p.C;
        const uint32_t dst = smem_u32(sA) + row_off;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int2 e = kt[j];
          const int sh = bh + (e.y >> 16), sw = bw + (e.y & 0xffff);
          const bool ok = row_ok && e.x >= 0 && sh >= 0 && sh < p.H && sw >= 0 && sw < p.W;
          const __nv_bfloat16* src = ok ? img + ((int64_t)sh * p.W + sw) * p.C + e.x : p.x;
          cp_async_16(dst + (((uint32_t)j ^ swz) << 4), src, ok ? 16u : 0u);
        }
        cp_async_commit();
        if (pend >= 0) {
          cp_async_wait<1>();
          fence_proxy_async_smem();
          mbar_arrive(&full[pend]);
        }
        pend = stage;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    cp_async_wait<0>();
    if (pend >= 0 && alive) {
      fence_proxy_async_smem();
      mbar_arrive(&full[pend]);
    }
  } else if (warp == 0) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc(1, 1, 1, true, true, CBM, WG_BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
        int tm, tn, kb0, kb1;
        unit_coords(u, tm, tn, kb0, kb1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * WG_BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t bBase = aBase + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < CBK / 16; ++k)
            mma_f16(d, make_sw128_desc(aBase + k * 2048, 8192, 1024), make_sw128_desc(bBase + k * 2048, 8192, 1024),
                    idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      int tm, tn, kb0, kb1;
      unit_coords(u, tm, tn, kb0, kb1);
      const int sp = u / per_split;
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int oc = tm * CBM + q * 32 + lane;
      float* dst = p.ws + ((int64_t)sp * p.OC + oc) * p.Kc;
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * WG_BN);
#pragma unroll 1
      for (int i = 0; i < WG_BN / 32; ++i) {
        uint32_t rr[32];
        tmem_ld32(tb + (uint32_t)(i * 32), rr);
        tmem_ld_wait();
        const int c0 = tn * WG_BN + i * 32;
        if (oc >= p.OC || c0 >= p.Kc) continue;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (c0 + j < p.Kc)  // Kc % 8 == 0: a 4-vector is entirely in or out
            *reinterpret_cast<float4*>(dst + c0 + j) =
                make_float4(__uint_as_float(rr[j]), __uint_as_float(rr[j + 1]), __uint_as_float(rr[j + 2]),
                            __uint_as_float(rr[j + 3]));
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// dW[oc][c][kh][kw] (+)= sum over splits of ws[split][oc][(kh*KW + kw)*C + c]
// (fixed split order: deterministic).
__global__ void wgrad_finish_kernel(const float* __restrict__ ws, int splits, int OC, int C, int KHW, float* __restrict__ dw,
                                    int accumulate) {
  const int64_t total = (int64_t)OC * C * KHW;
  const int Kc = KHW * C;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int oc = (int)(e / ((int64_t)C * KHW));
    const int rem = (int)(e - (int64_t)oc * C * KHW);
    const int c = rem / KHW, tap = rem - c * KHW;
    const int64_t col = (int64_t)tap * C + c;
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += ws[((int64_t)sp * OC + oc) * Kc + col];
    dw[e] = accumulate ? dw[e] + s : s;
  }
}

// Packs [OC][C][KH][KW] weights (fp32 or bf16) into the bf16 GEMM operand:
// forward   out[oc][(kh*KW + kw)*C + c]
// dgrad     out[c][(kh*KW + kw)*OC + oc]
// rows padded with zeros to Kpad columns.
template <typename T>
__global__ void conv_pack_weights_kernel(const T* __restrict__ w, __nv_bfloat16* __restrict__ out, int OC, int C,
                                         int KHW, int Kpad, int dgrad) {
  const int rows = dgrad ? C : OC;
  const int K = KHW * (dgrad ? OC : C);
  const int64_t total = (int64_t)rows * Kpad;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(e / Kpad), k = (int)(e - (int64_t)row * Kpad);
    float v = 0.f;
    if (k < K) {
      const int inner = dgrad ? OC : C;
      const int tap = k / inner, ch = k - tap * inner;
      const int oc = dgrad ? ch : row, c = dgrad ? row : ch;
      v = to_f32(w[((int64_t)oc * C + c) * KHW + tap]);
    }
    out[e] = __float2bfloat16_rn(v);
  }
}

int conv_tc_mode() {
  static int mode = [] {
    const char* e = std::getenv("DLVK_CONV_TC");
    return e ? std::atoi(e) : 0;
  }();
  return mode;
}
int g_conv_tc_override = -1;

template <int BN>
void launch_igemm(const CUtensorMap& tm, const IgemmParams& p, cudaStream_t s) {
  using C = IgCfg<BN>;
  static bool attr_set[kMaxDevices] = {false};
  const int dev = current_device_slot();
  if (!attr_set[dev]) {
    DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_igemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[dev] = true;
  }
  const int grid = std::min(p.tiles_m * p.tiles_n, tmap::sm_count());
  conv_igemm_kernel<BN><<<grid, IG_THREADS, C::SMEM, s>>>(tm, p);
  DLVK_POST_LAUNCH();
}

}  // namespace

// 0 = automatic (large bf16 convolutions), 1 = whenever supported, 2 = never.
void conv_tc_set_mode(int mode) { g_conv_tc_override = mode; }
int conv_tc_get_mode() { return g_conv_tc_override >= 0 ? g_conv_tc_override : conv_tc_mode(); }

bool conv2d_tc_supported(DType dt, const ConvDesc& d) {
  const int mode = conv_tc_get_mode();
  if (mode == 2 || dt != DType::BF16) return false;
  if (d.Cin % 8 != 0 || d.Cout % 8 != 0 || d.Cin < 16 || d.Cout < 16) return false;
  const int64_t khw = (int64_t)d.KH * d.KW;
  if (khw * d.Cin > (int64_t)KTAB_MAX * 8 || khw * d.Cout > (int64_t)KTAB_MAX * 8) return false;
  if (d.KH > 32767 || d.KW > 32767) return false;
  const int64_t P = (int64_t)d.N * d.Ho * d.Wo;
  if (P >= (1ll << 31) || (int64_t)d.N * d.H * d.W >= (1ll << 31)) return false;
  if (mode == 1) return true;
  const double flops = 2.0 * (double)P * d.Cout * (double)(khw * d.Cin);
  return flops >= 1.0e9;
}

int64_t conv_pack_cols(int64_t k) { return (k + CBK - 1) / CBK * CBK; }

void conv_pack_weights(DType wdt, const void* w, __nv_bfloat16* out, const ConvDesc& d, bool dgrad, cudaStream_t s) {
  const int KHW = d.KH * d.KW;
  const int Kpad = (int)conv_pack_cols((int64_t)KHW * (dgrad ? d.Cout : d.Cin));
  const int64_t total = (int64_t)(dgrad ? d.Cin : d.Cout) * Kpad;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  if (wdt == DType::F32)
    conv_pack_weights_kernel<float><<<grid, 256, 0, s>>>((const float*)w, out, d.Cout, d.Cin, KHW, Kpad, dgrad ? 1 : 0);
  else if (wdt == DType::BF16)
    conv_pack_weights_kernel<__nv_bfloat16>
        <<<grid, 256, 0, s>>>((const __nv_bfloat16*)w, out, d.Cout, d.Cin, KHW, Kpad, dgrad ? 1 : 0);
  else
    throw std::runtime_error("conv_pack_weights: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void conv2d_igemm(const __nv_bfloat16* src_nhwc, const __nv_bfloat16* wpack, const ConvDesc& d, bool dgrad,
                  const float* bias, bool relu, const void* mask, void* out, bool out_f32, cudaStream_t s) {
  IgemmParams p{};
  p.src = src_nhwc;
  if (!dgrad) {
    p.Hs = d.H, p.Ws = d.W, p.Cs = d.Cin;
    p.Ho = d.Ho, p.Wo = d.Wo;
    p.Ncols = d.Cout;
  } else {
    p.Hs = d.Ho, p.Ws = d.Wo, p.Cs = d.Cout;
    p.Ho = d.H, p.Wo = d.W;
    p.Ncols = d.Cin;
  }
  p.KW = d.KW;
  p.stride = d.stride;
  p.pad = d.pad;
  p.transposed = dgrad ? 1 : 0;
  p.P = d.N * p.Ho * p.Wo;
  p.K = d.KH * d.KW * p.Cs;
  const int Kpad = (int)conv_pack_cols(p.K);
  p.num_kb = Kpad / CBK;
  DLVK_CHECK(p.num_kb * 8 <= KTAB_MAX, "conv2d_igemm: filter too large");
  p.tiles_m = (p.P + CBM - 1) / CBM;
  p.out = out;
  p.out_f32 = out_f32 ? 1 : 0;
  p.bias = bias;
  p.relu = relu ? 1 : 0;
  p.mask = mask;
  p.err = device_error_word();
  tmap::bind_context();
  const int bn = p.Ncols <= 64 ? 64 : (p.Ncols <= 128 ? 128 : 256);
  p.tiles_n = (p.Ncols + bn - 1) / bn;
  const CUtensorMap tm = tmap::bf16_2d_sw128(wpack, (uint64_t)Kpad, (uint64_t)p.Ncols, (uint64_t)Kpad, (uint32_t)bn);
  if (bn == 64) launch_igemm<64>(tm, p, s);
  else if (bn == 128) launch_igemm<128>(tm, p, s);
  else launch_igemm<256>(tm, p, s);
}

static void wgrad_plan(const ConvDesc& d, int& tiles_m, int& tiles_n, int& num_kb, int& kbps, int& splits) {
  const int64_t P = (int64_t)d.N * d.Ho * d.Wo;
  const int Kc = d.KH * d.KW * d.Cin;
  tiles_m = (d.Cout + CBM - 1) / CBM;
  tiles_n = (Kc + WG_BN - 1) / WG_BN;
  num_kb = (int)((P + CBK - 1) / CBK);
  const int64_t work = (int64_t)num_kb * tiles_m * tiles_n;
  kbps = (int)std::max<int64_t>(8, (work + 2 * 148 - 1) / (2 * 148));
  kbps = std::min(kbps, num_kb);
  splits = (num_kb + kbps - 1) / kbps;
}

int64_t conv2d_wgrad_tc_ws_floats(const ConvDesc& d) {
  int tm, tn, nkb, kbps, splits;
  wgrad_plan(d, tm, tn, nkb, kbps, splits);
  return (int64_t)splits * d.Cout * d.KH * d.KW * d.Cin;
}

void conv2d_wgrad_tc(const __nv_bfloat16* x_nhwc, const __nv_bfloat16* dy_nhwc, const ConvDesc& d, float* ws,
                     float* dw, bool accumulate, cudaStream_t s) {
  WgradParams p{};
  p.x = x_nhwc;
  p.H = d.H, p.W = d.W, p.C = d.Cin;
  p.Ho = d.Ho, p.Wo = d.Wo, p.KW = d.KW, p.stride = d.stride, p.pad = d.pad;
  p.P = d.N * d.Ho * d.Wo;
  p.OC = d.Cout;
  p.Kc = d.KH * d.KW * d.Cin;
  wgrad_plan(d, p.tiles_m, p.tiles_n, p.num_kb, p.kb_per_split, p.splits);
  DLVK_CHECK(p.tiles_n * (WG_BN / 8) <= KTAB_MAX, "conv2d_wgrad_tc: filter too large");
  p.ws = ws;
  p.err = device_error_word();
  tmap::bind_context();
  // dY as a row-major [P, OC] matrix: 64 x 64 boxes, read M(OC)-major.
  const CUtensorMap tm = tmap::bf16_2d_sw128(dy_nhwc, (uint64_t)d.Cout, (uint64_t)p.P, (uint64_t)d.Cout, 64u);
  static bool attr_set[kMaxDevices] = {false};
  const int dev = current_device_slot();
  if (!attr_set[dev]) {
    DLVK_CUDA_CHECK(cudaFuncSetAttribute(conv_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, WgCfg::SMEM));
    attr_set[dev] = true;
  }
  const int units = p.tiles_m * p.tiles_n * p.splits;
  conv_wgrad_kernel<<<std::min(units, tmap::sm_count()), IG_THREADS, WgCfg::SMEM, s>>>(tm, p);
  DLVK_POST_LAUNCH();
  const int64_t total = (int64_t)d.Cout * d.Cin * d.KH * d.KW;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  wgrad_finish_kernel<<<grid, 256, 0, s>>>(ws, p.splits, d.Cout, d.Cin, d.KH * d.KW, dw, accumulate ? 1 : 0);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
