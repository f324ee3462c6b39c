// Tensor-core GEMM for sm_100a: TMA -> shared-memory ring -> tcgen05.mma ->
// TMEM accumulators -> fused epilogue.  Replaces the reference's
// matrix_multiply.comp / batch_matrix_multiply.comp (shaders/, dispatched from
// src/tensor/tensor_ops.cpp:187-298) for Dense forward/backward, attention
// projections and the batched attention products.
//
// Design:
//  * persistent kernel, one CTA per SM, 320 threads = 10 warps:
//      warp 0      TMA producer (one lane) over a STAGES-deep smem ring
//      warp 1      TMEM allocator + MMA issuer (one lane)
//      warps 2..9  epilogue: tcgen05.ld 32x32b -> alpha/beta/bias/act -> global
//  * tile 128 x BN x 64 (BN = 256 or 128), UMMA 128 x BN x 16 (kind::f16, bf16
//    in, f32 accumulate), two TMEM accumulator buffers so the epilogue of tile
//    i overlaps the main loop of tile i+1.
//  * A may be K-major ([M,K] row-major) or M-major ([K,M] row-major); B may be
//    K-major ([N,K]) or N-major ([K,N]).  Both are expressed through the TMA
//    box shape and the UMMA descriptor major-ness, so no transpose kernels are
//    ever needed for X*W, dY*W^T or X^T*dY.
//  * TMA loads are plain single-destination loads.
//  * every mbarrier wait is bounded (2 s) and reports through `err`.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/sm100.h"

namespace dlvk {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 elements per 128-byte swizzle row

struct TcParams {
  int M, N, K, batch;  // batch = number of (outer, inner) pairs
  int batch2;          // inner batch count
  int tiles_m, tiles_n;
  int a_mn, b_mn;
  void* C;
  int64_t ldc, bsc, bsc2;
  const void* R;       // residual (same dtype as C) or null
  int64_t ldr, bsr, bsr2;
  const void* Mk;      // ReLU mask source (same dtype as C) or null: out = 0 where Mk <= 0
  int64_t ldm, bsm, bsm2;
  int r_vec, m_vec;
  int out_f32;
  int vec_ok;
  float alpha, beta;
  const void* bias;
  int bias_f32;
  int act;
  uint32_t* err;
  int splits;          // split-K factor (1 = off); partials go to C (fp32 workspace)
  int kb_per_split;
  int64_t split_stride;  // elements between split slices of the workspace
  int i8;                  // 1: int8 x int8 -> int32 (kind::i8), K-major operands
  int tf32;                // 1: fp32 operands, tf32 math, fp32 accumulate (kind::tf32); single-CTA tiles
  const float* row_scale;  // int8 dequantisation: per-row (A) and per-column (B) scales
  const float* col_scale;
  float* colsum;           // per-32-row column sums of the output (staged fast path)
  int tma_c;               // 1: plain epilogue stores C through per-warp smem boxes + TMA;
                           // 2: same boxes, added into fp32 C (split-K partials reduced in L2)
  int a_bcast;             // 1: one A for every batch entry (its map has no batch extent)
  const float* row_bias;   // fp32 bias per output row, or null
  int sk;                  // 1: stream-K work split (fp32 C, partial tiles added by TMA reduces)
  uint32_t* bits_out;      // ReLU bitmask written (plain / TMA-store epilogues), or null
  const uint32_t* bits_in; // ReLU bitmask applied (staged epilogue), or null
  int64_t ldbits;          // 32-bit words per bitmask row
};

// PAIR: a 2-CTA cluster shares one 256 x BN tile (tcgen05 cta_group::2);
// each CTA stages its 128 rows of A and its BN/2 columns of B.
template <int BN, bool PAIR = false>
// BN = 512 (PAIR only): the tile is two N = 256 MMAs per k-step; each CTA
// stages two 128-column B sub-blocks, and the 512 accumulator columns fill
// TMEM, so there is one accumulator buffer instead of two.
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? (BN == 512 ? 4 : 6) : ((BN == 256) ? 4 : 6);
  static constexpr int ACCS = 2 * BN <= 512 ? 2 : 1;      // TMEM accumulator buffers
  static constexpr int TMEM_COLS = ACCS * BN;
  static constexpr int MMA_N = BN > 256 ? 256 : BN;        // N of one tcgen05.mma
  static constexpr int NSUB = BN / MMA_N;                  // MMAs per k-step
  static constexpr int SUB_B_BYTES = B_BYTES / NSUB;       // B bytes per sub-block
  static_assert(!(BN == 512) || PAIR, "the 512-column tile is a CTA-pair tile");
  // per-warp 32x33 fp32 staging; also holds the TMA-store boxes (8 x 4 KB
  // from the next 1024-byte boundary)
  static constexpr int EPI_BYTES = 8 * 32 * 33 * 4;
  static_assert(EPI_BYTES >= 768 + 8 * 4096, "epilogue smem too small for the TMA-store boxes");
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + EPI_BYTES;
  static_assert(SMEM <= 232448, "shared memory above the per-block limit");
  static_assert(STAGES * STAGE_BYTES / 8 >= 4096, "last-tile epilogue needs a 4 KB box per warp");
};

// Wait-time accounting for kernel development: compiled in only with
// DLVK_GEMM_TRACE defined (a standalone harness reads g_gemm_trace):
// per CTA, cycles spent waiting on each barrier class.
#ifdef DLVK_GEMM_TRACE
__device__ unsigned long long g_gemm_trace[148 * 16];
#define GEMM_T0() const long long _gt0 = clock64()
#define GEMM_ACC(slot) atomicAdd(&g_gemm_trace[blockIdx.x * 16 + (slot)], (unsigned long long)(clock64() - _gt0))
#define GEMM_STAMP(cond, slot)                                                              \
  do {                                                                                      \
    if (cond) g_gemm_trace[blockIdx.x * 16 + (slot)] = (unsigned long long)clock64();       \
  } while (0)
#else
#define GEMM_STAMP(cond, slot) \
  do {                         \
  } while (0)
#define GEMM_T0() \
  do {            \
  } while (0)
#define GEMM_ACC(slot) \
  do {                 \
  } while (0)
#endif

__device__ __forceinline__ void tile_coords(int t, const TcParams& p, int& tm, int& tn, int& b) {
  const int per_batch = p.tiles_m * p.tiles_n;
  b = t / per_batch;  // combined batch index; (outer, inner) = (b / batch2, b % batch2)
  const int r = t - b * per_batch;
  constexpr int GROUP_M = 8;
  const int in_group = GROUP_M * p.tiles_n;
  const int g = r / in_group;
  const int first_m = g * GROUP_M;
  const int gsz = min(p.tiles_m - first_m, GROUP_M);
  const int rr = r - g * in_group;
  tm = first_m + rr % gsz;
  tn = rr / gsz;
}

// The units of work of one CTA (or CTA pair) c of n.
//  - Tiles / split-K: unit t = (split, tile) for t = c, c + n, ...
//  - Stream-K (p.sk): the tiles x k-blocks iteration space is cut into n
//    equal contiguous ranges, one per CTA; the pieces of a range inside one
//    tile are its units (at most a few per CTA), each added into the fp32
//    output by the epilogue's TMA reduce, so no CTA idles in a last partial
//    wave.
// Producer, MMA issuer and epilogue each walk the same sequence.
struct WorkIter {
  int t;
  int64_t cur, hi;
};
__device__ __forceinline__ void work_begin(const TcParams& p, int c, int n, int num_kb, int tiles, WorkIter& w) {
  w.t = c;
  const int64_t total = (int64_t)tiles * num_kb;
  w.cur = total * c / n;
  w.hi = total * (c + 1) / n;
}
__device__ __forceinline__ bool work_next(const TcParams& p, int n, int num_kb, int tiles_per_split, int num_tiles,
                                          WorkIter& w, int& tm, int& tn, int& b, int& sp, int& kb0, int& kb1,
                                          bool& last) {
  if (p.sk) {
    if (w.cur >= w.hi) return false;
    const int tile = (int)(w.cur / num_kb);
    kb0 = (int)(w.cur - (int64_t)tile * num_kb);
    kb1 = (int)min((int64_t)num_kb, (int64_t)kb0 + (w.hi - w.cur));
    w.cur += kb1 - kb0;
    sp = 0;
    tile_coords(tile, p, tm, tn, b);
    last = w.cur >= w.hi;
    return true;
  }
  if (w.t >= num_tiles) return false;
  sp = w.t / tiles_per_split;
  tile_coords(w.t - sp * tiles_per_split, p, tm, tn, b);
  kb0 = sp * p.kb_per_split;
  kb1 = min(num_kb, kb0 + p.kb_per_split);
  last = w.t + n >= num_tiles;
  w.t += n;
  return true;
}

// Epilogue element loops below branch once per chunk, never per element: a
// per-element select between activation or bias variants inside a fully
// unrolled 32-wide loop is compiled to predicated code for every variant and
// made the epilogue, not the tensor cores, the bottleneck.
template <int VEC>
__device__ __forceinline__ void apply_act(int act, float* v) {
  if (act == ACT_RELU) {
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = fmaxf(v[k], 0.f);
  } else if (act == ACT_GELU) {
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = 0.5f * v[k] * (1.f + erff(v[k] * 0.70710678118654752f));
  }
}

template <int VEC>
__device__ __forceinline__ void add_bias(const void* bias, bool f32, int n, int valid, float* v) {
  if (f32) {
    const float* b = reinterpret_cast<const float*>(bias) + n;
    if (valid == VEC && (VEC % 4) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0) {
#pragma unroll
      for (int k = 0; k < VEC; k += 4) {
        const float4 t = *reinterpret_cast<const float4*>(b + k);
        v[k] += t.x;
        v[k + 1] += t.y;
        v[k + 2] += t.z;
        v[k + 3] += t.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k)
        if (k < valid) v[k] += b[k];
    }
  } else {
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(bias) + n;
#pragma unroll
    for (int k = 0; k < VEC; ++k)
      if (k < valid) v[k] += __bfloat162float(b[k]);
  }
}

// Row-per-lane epilogues (lane = row row0 + lane, v = its 32 columns from
// n0): zero v where the ReLU bitmask is clear, and rows past M entirely.
__device__ __forceinline__ void mask_row_bits(const TcParams& p, int row, int n0, float* v) {
  const uint32_t w = row < p.M ? p.bits_in[(int64_t)row * p.ldbits + (n0 >> 5)] : 0u;
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ((w >> j) & 1u) ? v[j] : 0.f;
}

// Column sums of a 32 x 32 chunk held one row per lane, by recursive
// halving: at each of five steps a lane keeps half of its columns and adds
// its partner's copies of them (16 + 8 + 4 + 2 + 1 shuffles), ending with
// lane l holding column l.  Written to the per-32-row partials
// colsum[(row0 / 32) * N + n].  Rows past M must be zero in v; v is consumed.
__device__ __forceinline__ void colsum_chunk(const TcParams& p, int row0, int lane, int n0, float* v) {
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {
    const bool up = (lane & h) != 0;
#pragma unroll
    for (int j = 0; j < h; ++j) {
      const float send = up ? v[j] : v[j + h];
      const float keep = up ? v[j + h] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  if (n0 + lane < p.N) p.colsum[(int64_t)(row0 >> 5) * p.N + n0 + lane] = v[0];
}

// v[j] += R[row, n0 + j] (bf16, C's dtype) for a row-per-lane epilogue: the
// lane reads its row's 32 consecutive elements as four 16-byte vectors.
__device__ __forceinline__ void add_row_residual(const TcParams& p, int64_t rb, int row, int n0, float* v) {
  if (row >= p.M || n0 >= p.N) return;
  const int64_t off = rb + (int64_t)row * p.ldr + n0;
  if (n0 + 32 <= p.N && p.r_vec) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.R) + off);
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) u[q] = src[q];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        v[8 * q + 2 * k] += f.x;
        v[8 * q + 2 * k + 1] += f.y;
      }
    }
  } else {
    for (int j = 0; j < 32 && n0 + j < p.N; ++j)
      v[j] += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.R)[off + j]);
  }
}

// Zero v[j] where the bf16 mask Mk[row, n0 + j] <= 0 (row-per-lane
// epilogue; the lane reads its row's 32 mask values as 16-byte vectors).
__device__ __forceinline__ void mask_row_bf16(const TcParams& p, int64_t mb, int row, int n0, float* v) {
  if (row >= p.M || n0 >= p.N) return;
  const int64_t off = mb + (int64_t)row * p.ldm + n0;
  if (n0 + 32 <= p.N && p.m_vec) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.Mk) + off);
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) u[q] = src[q];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[q]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        v[8 * q + 2 * k] = f.x > 0.f ? v[8 * q + 2 * k] : 0.f;
        v[8 * q + 2 * k + 1] = f.y > 0.f ? v[8 * q + 2 * k + 1] : 0.f;
      }
    }
  } else {
    for (int j = 0; j < 32 && n0 + j < p.N; ++j)
      if (!(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.Mk)[off + j]) > 0.f)) v[j] = 0.f;
  }
}

// Word of the ReLU bitmask for one row's 32 columns [n0, n0 + 32): bit j set
// where v[j] > 0 (after the activation); columns past N stay clear.
__device__ __forceinline__ void store_bits(const TcParams& p, int row, int n0, const float* v) {
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) w |= (v[j] > 0.f ? 1u : 0u) << j;
  if (p.N - n0 < 32) w &= (1u << (p.N - n0)) - 1u;
  p.bits_out[(int64_t)row * p.ldbits + (n0 >> 5)] = w;
}

template <typename T> __device__ __forceinline__ float ld_elem(const void* p, int64_t i) {
  return to_f32(reinterpret_cast<const T*>(p)[i]);
}

// Loads VEC consecutive elements of type T (VEC * sizeof(T) == 16 when `vec`).
template <typename T, int VEC>
__device__ __forceinline__ void ld_vec(const void* base, int64_t off, int valid, bool vec, float* out) {
  if (vec && valid == VEC) {
    uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(base) + off);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int k = 0; k < VEC; ++k) out[k] = to_f32(e[k]);
  } else {
#pragma unroll
    for (int k = 0; k < VEC; ++k) out[k] = k < valid ? ld_elem<T>(base, off + k) : 0.f;
  }
}

// Writes one staged 32x32 chunk: VEC columns per lane, 32/VEC lanes per row.
template <typename T, int VEC>
__device__ __forceinline__ void epi_store(const TcParams& p, const float* stg, int row0, int n0, int lane,
                                          int64_t cb, int64_t rb, int64_t mb) {
  constexpr int LPR = 32 / VEC;           // lanes per row
  constexpr int RPP = 32 / LPR;           // rows per pass
  constexpr int NP = 32 / RPP;            // passes
  const int cg = lane % LPR, rr = lane / LPR;
  const int n = n0 + cg * VEC;
  const int valid = max(0, min(VEC, p.N - n));
  // Fast path: whole 16-byte vectors everywhere.  All global reads of the
  // chunk (beta*C, residual, mask) are issued before any is consumed, so the
  // chunk pays one memory latency instead of one per pass.
  // ReLU bitmask: lane l loads the chunk's word of row row0 + l; the lanes
  // that handle a row take its bits with a shuffle.
  uint32_t bw = 0;
  if (p.bits_in) {
    const int r = row0 + lane;
    if (r < p.M && n0 < p.N) bw = p.bits_in[(int64_t)r * p.ldbits + (n0 >> 5)];
  }
  const int naux = (p.beta != 0.f) + (p.R != nullptr) + (p.Mk != nullptr);
  // Exactly one auxiliary input (beta*C, residual or mask) is prefetched; a
  // ReLU bitmask beside it takes the per-pass path below.
  const bool fast = naux == 1 && !p.bits_in && valid == VEC && p.vec_ok && (!p.R || p.r_vec) &&
                    (!p.Mk || p.m_vec) && row0 + 32 <= p.M;
  if (fast) {
    const T* abase;
    int64_t aoff, ald;
    if (p.beta != 0.f) {
      abase = reinterpret_cast<const T*>(p.C); aoff = cb; ald = p.ldc;
    } else if (p.R) {
      abase = reinterpret_cast<const T*>(p.R); aoff = rb; ald = p.ldr;
    } else {
      abase = reinterpret_cast<const T*>(p.Mk); aoff = mb; ald = p.ldm;
    }
    uint4 av[NP];
#pragma unroll
    for (int ps = 0; ps < NP; ++ps)
      av[ps] = *reinterpret_cast<const uint4*>(abase + aoff + (int64_t)(row0 + ps * RPP + rr) * ald + n);
    const int mode = p.beta != 0.f ? 0 : (p.R ? 1 : 2);
    float bv[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) bv[k] = 0.f;
    if (p.bias) add_bias<VEC>(p.bias, p.bias_f32, n, valid, bv);
    float cs[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) cs[k] = 0.f;
#pragma unroll
    for (int ps = 0; ps < NP; ++ps) {
      const int rl = ps * RPP + rr;
      float v[VEC];
      const float rbv = p.row_bias ? p.row_bias[row0 + rl] : 0.f;
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = stg[rl * 33 + cg * VEC + k] + bv[k] + rbv;
      const T* e = reinterpret_cast<const T*>(&av[ps]);
      if (mode == 0) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] += p.beta * to_f32(e[k]);
      } else if (mode == 1) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] += to_f32(e[k]);
      }
      apply_act<VEC>(p.act, v);
      if (mode == 2) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = to_f32(e[k]) > 0.f ? v[k] : 0.f;
      }
      uint4 u;
      T* eo = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int k = 0; k < VEC; ++k) eo[k] = from_f32<T>(v[k]);
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.C) + cb + (int64_t)(row0 + rl) * p.ldc + n) = u;
      if (p.colsum) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) cs[k] += v[k];
      }
    }
    if (p.colsum) {
      // The lanes with the same column group (lane % LPR) hold the other rows.
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
        for (int k = 0; k < VEC; ++k) cs[k] += __shfl_xor_sync(0xffffffffu, cs[k], off);
      if (rr == 0) {
        float* dst = p.colsum + (int64_t)(row0 >> 5) * p.N + n;
#pragma unroll
        for (int k = 0; k < VEC; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(cs[k], cs[k + 1], cs[k + 2], cs[k + 3]);
      }
    }
    return;
  }
#pragma unroll 1
  for (int pass = 0; pass < NP; ++pass) {
    const int rl = pass * RPP + rr;
    const int row = row0 + rl;
    const uint32_t mbits = p.bits_in ? (__shfl_sync(0xffffffffu, bw, rl) >> (cg * VEC)) : ~0u;
    if (row >= p.M || valid == 0) continue;
    float v[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = stg[rl * 33 + cg * VEC + k];
    const int64_t ci = cb + (int64_t)row * p.ldc + n;
    if (p.beta != 0.f) {
      float o[VEC];
      ld_vec<T, VEC>(p.C, ci, valid, p.vec_ok, o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] += p.beta * o[k];
    }
    if (p.bias) add_bias<VEC>(p.bias, p.bias_f32, n, valid, v);
    if (p.row_bias) {
      const float rbv = p.row_bias[row];
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] += rbv;
    }
    if (p.R) {
      float o[VEC];
      ld_vec<T, VEC>(p.R, rb + (int64_t)row * p.ldr + n, valid, p.r_vec, o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] += o[k];
    }
    apply_act<VEC>(p.act, v);
    if (p.Mk) {
      float o[VEC];
      ld_vec<T, VEC>(p.Mk, mb + (int64_t)row * p.ldm + n, valid, p.m_vec, o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = o[k] > 0.f ? v[k] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) v[k] = ((mbits >> k) & 1u) ? v[k] : 0.f;
    T* dst = reinterpret_cast<T*>(p.C) + ci;
    if (p.vec_ok && valid == VEC) {
      uint4 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int k = 0; k < VEC; ++k) e[k] = from_f32<T>(v[k]);
      *reinterpret_cast<uint4*>(dst) = u;
    } else {
      for (int k = 0; k < valid; ++k) dst[k] = from_f32<T>(v[k]);
    }
  }
}

// EPI = 1 compiles only the TMA-store epilogue (plain, bias, activation,
// bf16 residual or mask, bitmask, column sums, reduce-add): a kernel with a
// smaller instruction footprint for the common launches, whose epilogue
// otherwise misses in the instruction cache.  EPI = 2 is that path with
// alpha, bias and activation only.  EPI = 0 has every path.
template <int BN, bool PAIR = false, int EPI = 0>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, TcParams p) {
  using C = Cfg<BN, PAIR>;
  GEMM_STAMP(threadIdx.x == 0, 4);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  float* epi = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_per_split = p.tiles_m * p.tiles_n * p.batch;
  const int num_tiles = tiles_per_split * p.splits;  // work units
  // elements per 128-byte k-block: 64 bf16, 128 int8 or 32 fp32 (tf32)
  const int bke = p.i8 ? 2 * BK : (p.tf32 ? BK / 2 : BK);
  // M/N-major operands come as boxes of one 128-byte swizzle row along M/N
  // (64 bf16 or 32 fp32) by bke rows along K.
  const int mn_box = p.tf32 ? 32 : 64;
  const int mn_box_bytes = p.tf32 ? 4096 : 8192;
  const int num_kb = (p.K + bke - 1) / bke;
  // With PAIR the two CTAs of a cluster walk the same tiles; `rank` selects
  // the 128-row half of A / the BN/2-column half of B this CTA stages.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int t0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int TILE_M = PAIR ? 2 * BM : BM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      // PAIR: one arrival per epilogue warp of both CTAs (the leader's barrier
      // is the one the MMA warp waits on); otherwise one per epilogue thread.
      mbar_init(&tempty[i], PAIR ? 16 : 256);
    }
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs (our operands) are complete from here on
  GEMM_STAMP(threadIdx.x == 0, 5);

  if (warp == 0) {
    if (lane == 0 && PAIR) {
      int stage = 0;
      uint32_t phase = 0;
      WorkIter w;
      work_begin(p, t0, tstep, num_kb, tiles_per_split, w);
      int tm, tn, b, sp, kb0, kb1;
      bool last;
      while (work_next(p, tstep, num_kb, tiles_per_split, num_tiles, w, tm, tn, b, sp, kb0, kb1, last)) {
        const int bo = b / p.batch2, bi = b - bo * p.batch2;
        const int abo = p.a_bcast ? 0 : bo, abi = p.a_bcast ? 0 : bi;
        const int arow = tm * TILE_M + (int)rank * BM;
        // sub-block j of this CTA: columns tn*BN + j*MMA_N + rank*MMA_N/2 + [0, MMA_N/2)
        const int bcol = tn * BN + (int)rank * (C::MMA_N / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          {
            GEMM_T0();
            if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) goto producer_done_pair;
            GEMM_ACC(0);
          }
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);  // the leader's full barrier
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
          if (!p.a_mn) {
            tma_load_4d_pair(sA, &tmA, fb, kb * BK, arow, abi, abo);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_4d_pair(sA + j * 8192, &tmA, fb, arow + j * 64, kb * BK, abi, abo);
          }
#pragma unroll
          for (int sub = 0; sub < C::NSUB; ++sub) {
            uint8_t* sBs = sB + sub * C::SUB_B_BYTES;
            const int col = bcol + sub * C::MMA_N;
            if (!p.b_mn) {
              tma_load_4d_pair(sBs, &tmB, fb, kb * BK, col, bi, bo);
            } else {
#pragma unroll
              for (int j = 0; j < C::MMA_N / 128; ++j)
                tma_load_4d_pair(sBs + j * 8192, &tmB, fb, col + j * 64, kb * BK, bi, bo);
            }
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done_pair:;
    } else if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      WorkIter w;
      work_begin(p, blockIdx.x, gridDim.x, num_kb, tiles_per_split, w);
      int tm, tn, b, sp, kb0, kb1;
      bool last;
      while (work_next(p, gridDim.x, num_kb, tiles_per_split, num_tiles, w, tm, tn, b, sp, kb0, kb1, last)) {
        const int bo = b / p.batch2, bi = b - bo * p.batch2;
        const int abo = p.a_bcast ? 0 : bo, abi = p.a_bcast ? 0 : bi;
        for (int kb = kb0; kb < kb1; ++kb) {
          {
            GEMM_T0();
            if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) goto producer_done;
            GEMM_ACC(0);
          }
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if (!p.a_mn) {
            tma_load_4d(sA, &tmA, &full[stage], kb * bke, tm * BM, abi, abo);
          } else {
            for (int j = 0; j < BM / mn_box; ++j)
              tma_load_4d(sA + j * mn_box_bytes, &tmA, &full[stage], tm * BM + j * mn_box, kb * bke, abi, abo);
          }
          if (!p.b_mn) {
            tma_load_4d(sB, &tmB, &full[stage], kb * bke, tn * BN, bi, bo);
          } else {
            for (int j = 0; j < BN / mn_box; ++j)
              tma_load_4d(sB + j * mn_box_bytes, &tmB, &full[stage], tn * BN + j * mn_box, kb * bke, bi, bo);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && PAIR) {
      if (rank == 0) {
        // M = 256 across the pair; B descriptors describe this CTA's BN/2
        // columns (the peer's half sits at the same offsets in its smem).
        const uint32_t idesc = make_idesc(1, 1, 1, p.a_mn != 0, p.b_mn != 0, 2 * BM, C::MMA_N);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        WorkIter w;
        work_begin(p, t0, tstep, num_kb, tiles_per_split, w);
        int tm, tn, b, sp, kb0, kb1;
        bool last;
        while (work_next(p, tstep, num_kb, tiles_per_split, num_tiles, w, tm, tn, b, sp, kb0, kb1, last)) {
          {
            GEMM_T0();
            if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
            GEMM_ACC(1);
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(acc * BN);
          bool ok = true;
          for (int kb = kb0; kb < kb1; ++kb) {
            GEMM_T0();
            if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
            GEMM_ACC(2);
            tc_fence_after();
            const uint32_t aBase = smem_u32(smem + stage * C::STAGE_BYTES);
            const uint32_t bBase = aBase + C::A_BYTES;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t ad = p.a_mn ? make_sw128_desc(aBase + k * 2048, 8192, 1024)
                                         : make_sw128_desc(aBase + k * 32, 16, 1024);
#pragma unroll
              for (int sub = 0; sub < C::NSUB; ++sub) {
                const uint32_t bs = bBase + sub * C::SUB_B_BYTES;
                const uint64_t bd = p.b_mn ? make_sw128_desc(bs + k * 2048, 8192, 1024)
                                           : make_sw128_desc(bs + k * 32, 16, 1024);
                mma_f16_pair(d + (uint32_t)(sub * C::MMA_N), ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
              }
            }
            const uint32_t eb = smem_u32(&empty[stage]);
            mma_commit_pair(eb);
            mma_commit_pair(mapa_shared(eb, 1));
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          const uint32_t fb = smem_u32(&tfull[acc]);
          mma_commit_pair(fb);
          mma_commit_pair(mapa_shared(fb, 1));
          if (++acc == C::ACCS) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
    } else if (lane == 0) {
      const uint32_t idesc = p.i8 ? make_idesc(2, 1, 1, false, false, BM, BN)
                                  : (p.tf32 ? make_idesc(1, 2, 2, p.a_mn != 0, p.b_mn != 0, BM, BN)
                                            : make_idesc(1, 1, 1, p.a_mn != 0, p.b_mn != 0, BM, BN));
      // One MMA takes 32 bytes of K: a K-major operand advances 32 bytes per
      // MMA, an M/N-major one K rows of 128 bytes (16 bf16 / 8 tf32 rows).
      const uint32_t mn_step = p.tf32 ? 1024u : 2048u;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      WorkIter w;
      work_begin(p, blockIdx.x, gridDim.x, num_kb, tiles_per_split, w);
      int tm, tn, b, sp, kb0, kb1;
      bool last;
      while (work_next(p, gridDim.x, num_kb, tiles_per_split, num_tiles, w, tm, tn, b, sp, kb0, kb1, last)) {
        {
          GEMM_T0();
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
          GEMM_ACC(1);
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          GEMM_T0();
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          GEMM_ACC(2);
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t bBase = aBase + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // M/N-major tf32 operands use the 32-byte-atom swizzle (4-row atoms 512 bytes apart).
            const uint64_t ad = p.a_mn ? (p.tf32 ? make_sw128b32_desc(aBase + k * mn_step, (uint32_t)mn_box_bytes, 512)
                                                 : make_sw128_desc(aBase + k * mn_step, (uint32_t)mn_box_bytes, 1024))
                                       : make_sw128_desc(aBase + k * 32, 16, 1024);
            const uint64_t bd = p.b_mn ? (p.tf32 ? make_sw128b32_desc(bBase + k * mn_step, (uint32_t)mn_box_bytes, 512)
                                                 : make_sw128_desc(bBase + k * mn_step, (uint32_t)mn_box_bytes, 1024))
                                       : make_sw128_desc(bBase + k * 32, 16, 1024);
            if (p.i8) mma_i8(d, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else if (p.tf32) mma_tf32(d, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
            else mma_f16(d, ad, bd, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == C::ACCS) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // Epilogue warps 2..9: two warps per TMEM lane quarter (warp % 4), each
    // owning half of the tile's columns.  The TMEM load of the next 32-column
    // chunk is issued before the current chunk is processed.  Plain epilogues
    // (alpha, bias, activation) store straight from registers; with beta,
    // residual or ReLU mask the chunk is staged through shared memory so that
    // every extra global access is a coalesced 16-byte access along a row.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    float* stg = epi + ew * (32 * 33);
    // A bf16 residual and a bf16 ReLU mask are applied in registers; with
    // beta (or an fp32 output with either) the chunk goes through the staged
    // path, which handles all three.
    const bool staged = (p.beta != 0.f) || (p.out_f32 && (p.R != nullptr || p.Mk != nullptr));
    constexpr int NCH = BN / 64;  // 32-column chunks per warp
    int acc = 0, ecount = 0;
    uint32_t acc_phase = 0;
    // TMA-store boxes (4 KB): one slot per warp in the epilogue area, so each
    // box waits for the store issued before it.  A CTA's last tile has the
    // whole stage area to itself (every stage has been consumed by the MMAs
    // and no load is left), so there each warp gets 1/8 of it and issues its
    // boxes without waiting.
    constexpr int WREG = (C::STAGES * C::STAGE_BYTES / 8) & ~1023;
    WorkIter w;
    work_begin(p, t0, tstep, num_kb, tiles_per_split, w);
    int tm, tn, b, sp, kb0, kb1;
    bool last_tile;
    while (work_next(p, tstep, num_kb, tiles_per_split, num_tiles, w, tm, tn, b, sp, kb0, kb1, last_tile)) {
      int tcount = 0;  // boxes of this tile issued by this warp

      {
        GEMM_T0();
        if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
        if (threadIdx.x == 64) GEMM_ACC(3);
        GEMM_STAMP(threadIdx.x == 64 && g_gemm_trace[blockIdx.x * 16 + 6] == 0, 6);
        GEMM_STAMP(threadIdx.x == 64, 7);
      }
      tc_fence_after();
      const int bo = b / p.batch2, bi = b - bo * p.batch2;
      const int64_t cb = (int64_t)sp * p.split_stride + (int64_t)bo * p.bsc + (int64_t)bi * p.bsc2;
      const int64_t rb = (int64_t)bo * p.bsr + (int64_t)bi * p.bsr2;
      const int64_t mb = (int64_t)bo * p.bsm + (int64_t)bi * p.bsm2;
      const int row0 = tm * TILE_M + (int)rank * BM + q * 32;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + half * NCH * 32);
      uint32_t r[2][32];
      uint8_t* box = nullptr;  // the TMA-store box being filled
      tmem_ld32(tbase, r[0]);
      tmem_ld_wait();
      GEMM_STAMP(threadIdx.x == 64 && last_tile, 13);
      // Unrolled by two (the register double buffer needs the chunk parity at
      // compile time), not fully: eight full copies of the chunk body for the
      // 512-column tile make the epilogue's code large.
#pragma unroll 2
      for (int i = 0; i < NCH; ++i) {
        if (i == 1) GEMM_STAMP(threadIdx.x == 64 && last_tile, 15);
        if (i + 1 < NCH) tmem_ld32(tbase + (uint32_t)((i + 1) * 32), r[(i + 1) & 1]);
        const int n0 = tn * BN + (half * NCH + i) * 32;
        if (EPI == 0 && staged) {
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = __uint_as_float(r[i & 1][j]) * p.alpha;
          __syncwarp();
          if (n0 < p.N && row0 < p.M) {
            if (p.out_f32) epi_store<float, 4>(p, stg, row0, n0, lane, cb, rb, mb);
            else epi_store<__nv_bfloat16, 8>(p, stg, row0, n0, lane, cb, rb, mb);
          }
          __syncwarp();
        } else if (EPI == 1 || p.tma_c) {
          // Row `lane` of this warp's box goes to smem and one lane stores the
          // box with TMA (rows >= M / columns >= N are clipped).  fp32: one
          // 32 x 32 box (128-byte rows) per chunk.  bf16: chunks i, i+1 fill
          // the two halves of one 32 x 64 box, so every box row is a whole
          // 128-byte line and there is one store (and one proxy fence) per two
          // chunks.
          const bool bf = !p.out_f32;
          const bool opens = !bf || (i & 1) == 0;
          const int nbox = bf ? n0 - (i & 1) * 32 : n0;  // the box's first column
          if (nbox < p.N) {
            float v[32];
#pragma unroll
            const float rbv = (EPI != 2 && p.row_bias && row0 + lane < p.M) ? p.row_bias[row0 + lane] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(r[i & 1][j]), p.alpha, rbv);
            if (p.bias && n0 < p.N) add_bias<32>(p.bias, p.bias_f32, n0, min(32, p.N - n0), v);
            if (EPI != 2 && p.R) add_row_residual(p, rb, row0 + lane, n0, v);
            apply_act<32>(p.act, v);
            if (EPI != 2 && p.Mk) mask_row_bf16(p, mb, row0 + lane, n0, v);
            if (EPI != 2 && p.bits_in) mask_row_bits(p, row0 + lane, n0, v);
            if (EPI != 2 && p.bits_out && n0 < p.N && row0 + lane < p.M) store_bits(p, row0 + lane, n0, v);
            // Boxes start on 1024-byte boundaries (the swizzled box layout is
            // defined on aligned addresses).
            if (opens) {
              if (last_tile) {
                const int nslot = WREG / 4096;
                box = smem + ew * WREG + (tcount % nslot) * 4096;
                if (tcount > 0 && tcount % nslot == 0 && lane == 0) bulk_wait_group_read<0>();
              } else {
                box = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(epi) + 1023) & ~uintptr_t(1023)) +
                      ew * 4096;
                if (lane == 0) bulk_wait_group_read<0>();
              }
              __syncwarp();
            }
            // The box map uses the 128-byte swizzle, which the TMA unit applies
            // to shared-memory address bits: XOR the 16-byte chunk index with
            // address bits 7..9.
            const uint32_t bb = smem_u32(box) + (uint32_t)lane * 128u;
            if (!bf) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t a = bb + (uint32_t)j * 16u;
                st_shared_v4(a ^ (((a >> 7) & 7u) << 4), __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                             __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint32_t w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * j + 2 * k], v[8 * j + 2 * k + 1]);
                  w[k] = *reinterpret_cast<const uint32_t*>(&h);
                }
                const uint32_t a = bb + (uint32_t)((i & 1) * 4 + j) * 16u;
                st_shared_v4(a ^ (((a >> 7) & 7u) << 4), w[0], w[1], w[2], w[3]);
              }
            }
            if (BN != 512 && EPI != 2 && p.colsum) {  // after the box write: consumes v (512-wide tiles: never, see host)
              if (row0 + lane >= p.M) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = 0.f;
              }
              colsum_chunk(p, row0, lane, n0, v);
            }
            if (!bf || (i & 1)) {
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                if (p.tma_c == 2) tma_reduce_add_5d(&tmC, box, nbox, row0, bi, bo, 0);
                else tma_store_5d(&tmC, box, nbox, row0, bi, bo, sp);
                bulk_commit_group();
              }
              ++ecount;
              ++tcount;
            }
          }
        } else {
          const int row = row0 + lane;
          if (row < p.M && n0 < p.N) {
            float v[32];
            const float rbv = p.row_bias ? p.row_bias[row] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(r[i & 1][j]), p.alpha, rbv);
            if (p.i8) {
              // int32 accumulators -> real values: alpha * acc * row_scale * col_scale
              const float rs = p.alpha * p.row_scale[row];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = (float)(int)r[i & 1][j] * rs;
              float cs[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) cs[j] = 0.f;
              add_bias<32>(p.col_scale, true, n0, min(32, p.N - n0), cs);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] *= cs[j];
            }
            if (p.bias) add_bias<32>(p.bias, p.bias_f32, n0, min(32, p.N - n0), v);
            if (p.R) add_row_residual(p, rb, row, n0, v);
            apply_act<32>(p.act, v);
            if (p.Mk) mask_row_bf16(p, mb, row, n0, v);
            if (p.bits_in) mask_row_bits(p, row, n0, v);
            if (p.bits_out) store_bits(p, row, n0, v);
            const bool full = (n0 + 32 <= p.N) && p.vec_ok;
            if (p.out_f32) {
              float* dst = reinterpret_cast<float*>(p.C) + cb + (int64_t)row * p.ldc + n0;
              if (full) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < p.N) dst[j] = v[j];
              }
            } else {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + cb + (int64_t)row * p.ldc + n0;
              if (full) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint4 u;
                  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
                  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[8 * j + 2 * k], v[8 * j + 2 * k + 1]);
                  reinterpret_cast<uint4*>(dst)[j] = u;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (n0 + j < p.N) dst[j] = __float2bfloat16_rn(v[j]);
              }
            }
          }
        }
        if (i + 1 < NCH) tmem_ld_wait();
      }
      GEMM_STAMP(threadIdx.x == 64 && last_tile, 14);
      tc_fence_before();
      if (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      } else {
        mbar_arrive(&tempty[acc]);
      }
      if (++acc == C::ACCS) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (p.tma_c && lane == 0) bulk_wait_group_read<0>();  // the boxes' smem is read before the CTA exits
  }
  GEMM_STAMP(threadIdx.x == 64, 9);
  GEMM_STAMP(threadIdx.x == 32, 11);
  GEMM_STAMP(threadIdx.x == 0, 12);
  tc_fence_before();
  __syncthreads();
  GEMM_STAMP(threadIdx.x == 64, 8);
  if (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  GEMM_STAMP(threadIdx.x == 64, 10);
  pdl_trigger();             // this CTA's work is done: the next kernel may start launching
  if (warp == 1) {
    tc_fence_after();
    if (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor-map encoding through the driver entry point (no libcuda
// link dependency), cached per device.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    DLVK_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || ptr == nullptr)
      throw std::runtime_error("dlvk: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D operand tensor map: dims {d0 (contiguous), d1, inner batch, outer
// batch}, strides in elements, box {one 128-byte row, box1, 1, 1}, 128-byte
// swizzle, zero fill out of bounds.
// Operand element kinds of the tensor maps.
enum class Elem { BF16, I8, F32 };

CUtensorMap make_tmap(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1, uint64_t s2,
                      uint64_t s3, uint32_t box1, Elem el, bool mn_major = false) {
  CUtensorMap m;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  const uint64_t esz = el == Elem::I8 ? 1 : (el == Elem::F32 ? 4 : 2);
  cuuint64_t strides[3] = {s1 * esz, s2 * esz, s3 * esz};
  cuuint32_t box[4] = {(cuuint32_t)(128 / esz), box1, 1, 1};  // one 128-byte swizzle row
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = el == Elem::I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                : (el == Elem::F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  CUresult r = encode_fn()(&m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           (el == Elem::F32 && mn_major) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                                         : CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("dlvk: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

int sm_count() {
  static int n[kMaxDevices] = {0};
  const int dev = current_device_slot();
  if (n[dev] == 0) DLVK_CUDA_CHECK(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return n[dev];
}

// The epilogue paths a launch needs: 1 = TMA-store path only (its C map was
// made and no input is staged through shared memory), 0 = all paths.
int epi_kind(const TcParams& p) {
  const bool staged = (p.beta != 0.f) || (p.out_f32 && (p.R != nullptr || p.Mk != nullptr));
  if (p.tma_c == 0 || staged) return 0;
  const bool extras = p.R || p.Mk || p.bits_in || p.bits_out || p.colsum || p.row_bias;
  static const bool plain_on = [] { const char* e = std::getenv("DLVK_GEMM_EPI2"); return !(e && e[0] == '0'); }();
  return (extras || !plain_on) ? 1 : 2;
}

template <int BN, int EPI>
void launch_tc_k(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& p, int max_ctas,
                 cudaStream_t s) {
  using C = Cfg<BN>;
  static bool attr_set[kMaxDevices] = {false};
  const int dev = current_device_slot();
  if (!attr_set[dev]) {
    DLVK_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_tc_kernel<BN, false, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n * p.batch * p.splits;
  const int slots = max_ctas > 0 ? max_ctas : sm_count();
  int grid = p.sk ? slots : std::min(tiles, slots);  // stream-K: every CTA takes a share
  launch_pdl(gemm_tc_kernel<BN, false, EPI>, dim3(grid), dim3(320), C::SMEM, s, ta, tb, tc, p);
  DLVK_POST_LAUNCH();
}
template <int BN>
void launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& p, int max_ctas,
               cudaStream_t s) {
  const int k = epi_kind(p);
  if (k == 2) launch_tc_k<BN, 2>(ta, tb, tc, p, max_ctas, s);
  else if (k == 1) launch_tc_k<BN, 1>(ta, tb, tc, p, max_ctas, s);
  else launch_tc_k<BN, 0>(ta, tb, tc, p, max_ctas, s);
}

// 2-CTA clusters sharing 256 x BN tiles (cta_group::2).  The persistent
// grid is as many pairs as can be resident at once.
template <int BN, int EPI>
void launch_tc_pair_k(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& p,
                      int max_ctas, cudaStream_t s) {
  using C = Cfg<BN, true>;
  static int max_pairs[kMaxDevices] = {0};
  const int dev = current_device_slot();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.blockDim = dim3(320, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // occupancy query: cluster shape only
  if (max_pairs[dev] == 0) {
    DLVK_CUDA_CHECK(
        cudaFuncSetAttribute(gemm_tc_kernel<BN, true, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    cfg.gridDim = dim3(2 * 74, 1, 1);
    int n = 0;
    DLVK_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, true, EPI>, &cfg));
    max_pairs[dev] = std::max(1, n);
  }
  const int tiles = p.tiles_m * p.tiles_n * p.batch * p.splits;
  int pairs = p.sk ? max_pairs[dev] : std::min(tiles, max_pairs[dev]);  // stream-K: every pair takes a share
  if (max_ctas > 0) pairs = std::max(1, std::min(pairs, max_ctas / 2));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.numAttrs = 2;
  DLVK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, true, EPI>, ta, tb, tc, p));
  DLVK_POST_LAUNCH();
}
template <int BN>
void launch_tc_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& p,
                    int max_ctas, cudaStream_t s) {
  const int k = epi_kind(p);
  if (k == 2) launch_tc_pair_k<BN, 2>(ta, tb, tc, p, max_ctas, s);
  else if (k == 1) launch_tc_pair_k<BN, 1>(ta, tb, tc, p, max_ctas, s);
  else launch_tc_pair_k<BN, 0>(ta, tb, tc, p, max_ctas, s);
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Split-K reduction: C = act(alpha * sum_s W[s] + beta * C + bias + R), masked.
// W is the fp32 workspace [splits][batch][M][N]; summation is in split order
// (deterministic).  One thread per output element.
template <typename T>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t per_split, GemmArgs a) {
  const int64_t MN = a.M * a.N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_split;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) acc += ws[s2 * per_split + i];
    const int64_t b = i / MN, r = i - b * MN;
    const int64_t m = r / a.N, n = r - m * a.N;
    const int64_t bo = b / a.batch2, bi = b - bo * a.batch2;
    T* c = reinterpret_cast<T*>(a.C) + bo * a.batch_stride_c + bi * a.batch2_stride_c + m * a.ldc + n;
    float v = a.alpha * acc;
    if (a.beta != 0.f) v += a.beta * to_f32(*c);
    if (a.bias)
      v += a.bias_dtype == (int)DType::F32 ? reinterpret_cast<const float*>(a.bias)[n]
                                           : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[n]);
    if (a.row_bias) v += a.row_bias[m];
    if (a.residual)
      v += to_f32(reinterpret_cast<const T*>(a.residual)[bo * a.batch_stride_r + bi * a.batch2_stride_r + m * a.ldr + n]);
    if (a.act == ACT_RELU) v = fmaxf(v, 0.f);
    else if (a.act == ACT_GELU) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    if (a.relu_mask &&
        !(to_f32(reinterpret_cast<const T*>(a.relu_mask)[bo * a.batch_stride_m + bi * a.batch2_stride_m + m * a.ldm + n]) >
          0.f))
      v = 0.f;
    if (a.relu_bits && !((a.relu_bits[m * a.ldbits + (n >> 5)] >> (n & 31)) & 1u)) v = 0.f;

    *c = from_f32<T>(v);
  }
}

// Tile shape and split-K choice from a small time model: per-SM tensor rate
// ~8 TFLOP/s at BN = 256 (15% less at BN = 128, which reloads A twice as
// often per FLOP), whole waves of persistent CTAs, and for split-K the fp32
// workspace write + read at ~5 TB/s plus one extra launch.
// Picks the tile shape, the split-K factor and whether the CTA-pair kernel
// runs, by a wave model: time = waves x (per-unit MMA time at an efficiency
// measured for that tile shape) + the split-K partial traffic.  Pair units
// are 256 x 256 tiles on sms/2 pairs (about 1.2x the single-CTA 128 x 256
// rate on B200); single units are 128 x BN on sms CTAs.
// The 256 x 512 pair tile: 0 never, 1 when the model picks it (default),
// 2 whenever it applies (measurement).  DLVK_GEMM_WIDE or gemm_tc_set_wide.
int& wide_flag() {
  static int f = [] {
    const char* e = std::getenv("DLVK_GEMM_WIDE");
    return e ? std::atoi(e) : 1;
  }();
  return f;
}
bool gemm_tc_wide_enabled() { return wide_flag() != 0; }
// With `red` (split_red_ok) the partials are added into C by the epilogue's
// TMA reduce in L2 (plus a clear of C when beta = 0) instead of the workspace
// round trip and the reduce launch.
// DLVK_GEMM_STREAMK: 0 never, 1 when the tiling model picks it (default),
// 2 whenever the output allows it (measurement).
int streamk_mode() {
  static const int m = [] {
    const char* e = std::getenv("DLVK_GEMM_STREAMK");
    return e ? std::atoi(e) : 1;
  }();
  return m;
}

void choose_tiling(const GemmArgs& a, int sms, int& BN, int& splits, bool& pair, bool red = false,
                   bool out_f32 = false, bool single_cta = false, bool* sk = nullptr) {
  if (sk) *sk = false;
  const int64_t kbs = (a.K + BK - 1) / BK;
  const double sm_flops = 8.1e12;
  double best = 1e300;
  BN = 256;
  splits = 1;
  pair = false;
  const bool pair_ok = !single_cta && gemm_tc_pair_enabled() && a.M >= 256 && sms >= 2;
  struct Cand {
    bool pair;
    int bn;
    double eff;
  };
  // The 256 x 512 pair tile moves 25% fewer L2 bytes per FLOP than 256 x 256
  // (the mainloop of the latter waits on L2 ~25% of the time), but its single
  // TMEM buffer leaves every tile's epilogue exposed.
  // Measured per-SM rates relative to the single-CTA tile: the wide tile's
  // mainloop runs ~1 090 cycles per 64-deep k-block (1.75x) below K = 8192
  // (back-to-back timings of 8192 x 1024 x {1024, 3072, 4096} against the
  // 256-wide pair tile), and 1.55x is kept from K = 8192 on.
  const double wide_eff = kbs >= 128 ? 1.55 : 1.75;
  const Cand cands[] = {{true, 512, wide_eff}, {true, 256, 1.2}, {false, 256, 1.0}, {false, 128, 0.85}};
  for (const Cand& c : cands) {
    if (c.pair && !pair_ok) continue;
    if (c.bn == 512 && (!gemm_tc_wide_enabled() || a.N < 512)) continue;
    if (c.bn != 512 && wide_flag() == 2 && pair_ok && a.N >= 512 && best < 1e300) continue;
    if (c.bn == 256 && a.N < 256) continue;
    const int64_t tile_m = c.pair ? 2 * BM : BM;
    const int64_t tiles = ((a.M + tile_m - 1) / tile_m) * ((a.N + c.bn - 1) / c.bn) * a.batch * a.batch2;
    const int64_t slots = c.pair ? sms / 2 : sms;
    for (int sp : {1, 2, 3, 4, 6, 8}) {
      if (sp > 1 && kbs / sp < 8) break;
      const int64_t units = tiles * sp;
      const int64_t waves = (units + slots - 1) / slots;
      const double unit_s = (double)tile_m * c.bn * BK * 2.0 * ((kbs + sp - 1) / sp) /
                            (sm_flops * (c.pair ? 2 : 1) * c.eff);
      // Epilogue of one CTA's 128 x BN block (measured: ~17 GB/s per CTA for
      // 128 x 256, ~18 GB/s for 128 x 512), exposed once at the end, or
      // after every wave without a second accumulator buffer.
      const double epi_s = 128.0 * c.bn * ((out_f32 || sp > 1) ? 4.0 : 2.0) / (c.bn == 512 ? 18e9 : 17e9);
      double t = waves * unit_s + (c.bn == 512 ? waves : 1) * epi_s;
      if (sp > 1) {
        const double mn = (double)a.M * a.N * a.batch * a.batch2;
        t += red ? sp * mn * 4.0 / 8e12 + (a.beta == 0.f ? mn * 4.0 / 5e12 + 2e-6 : 0.0)
                 : sp * mn * 8.0 / 5e12 + 5e-6;
      }
      if (t < best * 0.97) {
        best = t;
        BN = c.bn;
        splits = sp;
        pair = c.pair;
        if (sk) *sk = false;
      }
    }
    // Stream-K (fp32 C with a linear epilogue): every slot gets the same
    // number of k-blocks; a slot's pieces of about two tiles are added into C
    // by TMA reduces (each slot's last epilogue is exposed), after a clear of
    // C when beta = 0.
    if (sk && red && c.bn != 512 && streamk_mode() != 0) {
      const int64_t total = tiles * kbs;
      const int64_t per = (total + slots - 1) / slots;
      const double kb_s = (double)tile_m * c.bn * BK * 2.0 / (sm_flops * (c.pair ? 2 : 1) * c.eff);
      const double mn = (double)a.M * a.N * a.batch * a.batch2;
      const double t = per * kb_s + 2.0 * 128.0 * c.bn * 4.0 / 17e9 +
                       (double)(tiles + slots) * tile_m * c.bn * 4.0 / 8e12 +
                       (a.beta == 0.f ? mn * 4.0 / 5e12 + 2e-6 : 0.0);
      if (t < best * 0.97 || (streamk_mode() == 2 && !*sk)) {
        best = t;
        BN = c.bn;
        splits = 1;
        pair = c.pair;
        *sk = true;
      }
    }
  }
}

}  // namespace

namespace {
// DLVK_GEMM_TMA_STORE=0 keeps the register-direct epilogue stores.
bool tma_c_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("DLVK_GEMM_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return on;
}
// DLVK_GEMM_SPLITK_RED=0 keeps split-K on the workspace + reduce-kernel path,
// whose summation order is fixed (bitwise reproducible run to run).
bool split_red_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("DLVK_GEMM_SPLITK_RED");
    return !(e && e[0] == '0');
  }();
  return on;
}
// Split-K partials can be added straight into C: fp32 C without batching,
// an epilogue that is linear in the accumulator (alpha only; beta 0 or 1),
// and the alignment the fp32 C map needs.
bool split_red_ok(DType out_dt, const GemmArgs& a) {
  return split_red_enabled() && tma_c_enabled() && out_dt == DType::F32 && a.batch == 1 && a.batch2 == 1 &&
         (a.beta == 0.f || a.beta == 1.f) && a.bias == nullptr && a.residual == nullptr &&
         a.relu_mask == nullptr && a.relu_bits == nullptr && a.relu_bits_out == nullptr && a.act == ACT_NONE &&
         al16(a.C) && (a.ldc * 4) % 16 == 0 &&
         a.ldc * 4 < (1LL << 40) && a.N % 4 == 0;
}
}  // namespace

// The column sums come from the staged epilogue's fast path, which must
// then cover every chunk: exactly one auxiliary input (beta * C, residual or
// ReLU mask) with 16-byte rows, M and N multiples of 32 (every lane of a
// warp takes the fast path, so the lane shuffles are uniform), no
// batching.
bool gemm_tc_colsum_ok(DType out_dt, const GemmArgs& a) {
  const int esz = out_dt == DType::F32 ? 4 : 2;
  const int naux = (a.beta != 0.f) + (a.residual != nullptr) + (a.relu_mask != nullptr);
  auto rows16 = [&](const void* p, int64_t ld) {
    return p == nullptr || (al16(p) && (ld * esz) % 16 == 0);
  };
  // Staged epilogues (beta, or an fp32 output with a residual or mask) sum
  // their transposed chunk on the fast path (exactly one such input); the
  // others sum in registers on the TMA-store path.
  const bool staged = a.beta != 0.f || (out_dt == DType::F32 && (a.residual != nullptr || a.relu_mask != nullptr));
  return (staged ? naux == 1 : tma_c_enabled()) && a.batch == 1 && a.batch2 == 1 && a.M % 32 == 0 &&
         a.N % 32 == 0 && al16(a.C) &&
         (a.ldc * esz) % 16 == 0 && rows16(a.residual, a.ldr) && rows16(a.relu_mask, a.ldm);
}

bool gemm_tc_supported(const GemmArgs& a) {
  const bool a_k = (a.sak == 1), a_m = (a.sam == 1) && !a_k;
  const bool b_k = (a.sbk == 1), b_n = (a.sbn == 1) && !b_k;
  if (!(a_k || a_m) || !(b_k || b_n)) return false;
  const int64_t lda = a_k ? a.sam : a.sak;
  const int64_t ldb = b_k ? a.sbn : a.sbk;
  if ((lda * 2) % 16 || (ldb * 2) % 16) return false;
  if (a.batch > 1 && ((a.batch_stride_a * 2) % 16 || (a.batch_stride_b * 2) % 16)) return false;
  if (a.batch2 > 1 && ((a.batch2_stride_a * 2) % 16 || (a.batch2_stride_b * 2) % 16)) return false;
  if (a.batch * a.batch2 * ((a.M + 127) / 128) * ((a.N + 127) / 128) > (1LL << 31) - 1) return false;
  if (!al16(a.A) || !al16(a.B)) return false;
  if (a.M < 1 || a.N < 16 || a.K < 1) return false;
  if (a.M > (1LL << 31) - 1 || a.N > (1LL << 31) - 1 || a.K > (1LL << 31) - 1) return false;
  return true;
}

namespace {
// Plain epilogues (alpha, bias, activation; split-K partials included) store
// C with TMA from per-warp 32 x 32 boxes: one async bulk store per box
// instead of each lane writing its own row (32 scattered 16-byte stores per
// warp instruction).  The map is 5-D {N, M, inner batch, outer batch, split}
// with the epilogue's strides; sets p.tma_c when it applies.
CUtensorMap make_c_map(TcParams& p, int64_t M, int64_t N, bool reduce = false) {
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  p.tma_c = 0;
  // A bf16 residual or ReLU mask is applied in registers on this path; with
  // an fp32 output either one (and beta) takes the staged epilogue instead.
  if ((p.out_f32 && (p.R != nullptr || p.Mk != nullptr)) || p.beta != 0.f || p.i8 || !p.vec_ok || !tma_c_enabled())
    return tc;
  const uint64_t esz = p.out_f32 ? 4 : 2;
  auto pick = [&](int64_t cnt, int64_t stride) -> uint64_t {
    return cnt > 1 ? (uint64_t)stride * esz : (uint64_t)M * (uint64_t)p.ldc * esz;
  };
  const int64_t batch_outer = p.batch / p.batch2;
  const int64_t slices = reduce ? 1 : p.splits;  // reduce: every split adds into the one C
  cuuint64_t dims[5] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)p.batch2, (cuuint64_t)batch_outer,
                        (cuuint64_t)slices};
  cuuint64_t strides[4] = {(cuuint64_t)p.ldc * esz, pick(p.batch2, p.bsc2), pick(batch_outer, p.bsc),
                           pick(slices, p.split_stride)};
  for (uint64_t st : strides)
    if (st == 0 || st % 16 != 0 || st >= (1ull << 40)) return tc;
  cuuint32_t box[5] = {p.out_f32 ? 32u : 64u, 32u, 1u, 1u, 1u};  // 128-byte rows
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = encode_fn()(&tc, p.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, p.C,
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) p.tma_c = reduce ? 2 : 1;
  return tc;
}
}  // namespace

namespace {
// Tiling forced by gemm_tc_set_tiling (measurement only; 0 / -1 = the model's choice).
struct TilingOverride {
  int bn = 0, splits = 0, pair = -1;
};
TilingOverride& tiling_override() {
  static TilingOverride t;
  return t;
}
}  // namespace

void gemm_tc_set_tiling(int bn, int splits, int pair) {
  tiling_override() = TilingOverride{bn, splits, pair};
}

namespace {
// Shared host path of the bf16 and the tf32 GEMM.  TF32 runs on single-CTA
// tiles (no CTA pairs): fp32 operands, 32-element k-blocks.
void gemm_tc_impl(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas, float* workspace,
                  int64_t workspace_floats, bool tf32) {
  const Elem el = tf32 ? Elem::F32 : Elem::BF16;
  const int bke = tf32 ? BK / 2 : BK;
  if (a.M == 0 || a.N == 0) return;
  // The tensor-map encoder is a driver call and needs a current context on
  // this thread.  Threads that have only used the runtime through a "same
  // device" cudaSetDevice shortcut (e.g. PyTorch's autograd workers) may not
  // have one yet, so bind the primary context once per thread and device.
  {
    thread_local int bound_dev = -1;
    int dev = 0;
    DLVK_CUDA_CHECK(cudaGetDevice(&dev));
    if (bound_dev != dev) {
      DLVK_CUDA_CHECK(cudaSetDevice(dev));
      bound_dev = dev;
    }
  }
  const bool a_k = (a.sak == 1);
  const bool b_k = (a.sbk == 1);
  int BN = 256, splits = 1;
  bool pair = false, sk = false;
  const bool red = split_red_ok(out_dt, a);
  choose_tiling(a, max_ctas > 0 ? max_ctas : sm_count(), BN, splits, pair, red, out_dt == DType::F32, tf32, &sk);
  {
    const TilingOverride& ov = tiling_override();
    if (ov.pair >= 0) pair = ov.pair != 0 && !tf32 && a.M >= 256;
    if (ov.bn > 0) BN = (ov.bn == 512 && !pair) ? 256 : ov.bn;
    if (ov.splits > 0) {
      splits = ov.splits;
      sk = false;
    } else if (ov.splits == -1) {  // stream-K
      splits = 1;
      sk = red;
    }
  }
  if (BN == 512) sk = false;
  if (a.colsum != nullptr) {
    DLVK_CHECK(gemm_tc_colsum_ok(out_dt, a), "gemm_tc: column sums need the staged fast-path layout");
    splits = 1;  // the sums are taken over final outputs
    // without a staged input the TMA-store epilogue sums in registers, which
    // the 512-wide tile's instantiation leaves out (register budget)
    if (BN == 512 && a.beta == 0.f && !(out_dt == DType::F32 && (a.residual != nullptr || a.relu_mask != nullptr)))
      BN = 256;
  }
  if (a.relu_bits != nullptr || a.relu_bits_out != nullptr)
    DLVK_CHECK(a.batch == 1 && a.batch2 == 1 && a.ldbits >= (a.N + 31) / 32, "gemm_tc: ReLU bitmask needs a 2-D GEMM");
  if (a.relu_bits_out != nullptr) {
    DLVK_CHECK(a.residual == nullptr && a.relu_mask == nullptr && a.relu_bits == nullptr && a.beta == 0.f,
               "gemm_tc: the ReLU bitmask is written by plain epilogues only");
    splits = 1;  // the bits are taken from final outputs
  }
  if (!red && (workspace == nullptr || workspace_floats < (int64_t)splits * a.M * a.N * a.batch * a.batch2))
    splits = 1;
  if (a.colsum != nullptr || a.relu_bits_out != nullptr || !red) sk = false;
  pair = pair && max_ctas != 1;
  // Unused batch levels get a harmless stride (a multiple of 16 bytes).
  auto pick = [](int64_t cnt, int64_t stride, uint64_t dflt) { return cnt > 1 ? (uint64_t)stride : dflt; };
  CUtensorMap ta, tb;
  // A shared by every batch entry (zero batch strides): its map covers one
  // matrix and the producer reads it at batch coordinate 0.
  const bool a_bcast = a.batch * a.batch2 > 1 && (a.batch == 1 || a.batch_stride_a == 0) &&
                       (a.batch2 == 1 || a.batch2_stride_a == 0);
  const uint64_t ab2 = a_bcast ? 1 : (uint64_t)a.batch2, ab = a_bcast ? 1 : (uint64_t)a.batch;
  if (a_k) {
    const uint64_t d = (uint64_t)a.sam * (uint64_t)a.M;
    ta = make_tmap(a.A, a.K, a.M, ab2, ab, a.sam, pick((int64_t)ab2, a.batch2_stride_a, d),
                   pick((int64_t)ab, a.batch_stride_a, d), BM, el);
  } else {
    const uint64_t d = (uint64_t)a.sak * (uint64_t)a.K;
    ta = make_tmap(a.A, a.M, a.K, ab2, ab, a.sak, pick((int64_t)ab2, a.batch2_stride_a, d),
                   pick((int64_t)ab, a.batch_stride_a, d), (uint32_t)bke, el, true);
  }
  if (b_k) {
    const uint64_t d = (uint64_t)a.sbn * (uint64_t)a.N;
    tb = make_tmap(a.B, a.K, a.N, a.batch2, a.batch, a.sbn, pick(a.batch2, a.batch2_stride_b, d),
                        pick(a.batch, a.batch_stride_b, d), pair ? 128 : BN, el);
  } else {
    const uint64_t d = (uint64_t)a.sbk * (uint64_t)a.K;
    tb = make_tmap(a.B, a.N, a.K, a.batch2, a.batch, a.sbk, pick(a.batch2, a.batch2_stride_b, d),
                        pick(a.batch, a.batch_stride_b, d), (uint32_t)bke, el, true);
  }
  TcParams p{};
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.batch = (int)(a.batch * a.batch2);
  p.batch2 = (int)a.batch2;
  p.tiles_m = (int)((a.M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
  p.tiles_n = (int)((a.N + BN - 1) / BN);
  p.a_mn = a_k ? 0 : 1;
  p.b_mn = b_k ? 0 : 1;
  p.C = a.C;
  p.ldc = a.ldc;
  p.bsc = a.batch_stride_c;
  p.bsc2 = a.batch2_stride_c;
  p.R = a.residual;
  p.ldr = a.ldr;
  p.bsr = a.batch_stride_r;
  p.bsr2 = a.batch2_stride_r;
  p.Mk = a.relu_mask;
  p.ldm = a.ldm;
  p.bsm = a.batch_stride_m;
  p.bsm2 = a.batch2_stride_m;
  p.out_f32 = (out_dt == DType::F32);
  const int esz = p.out_f32 ? 4 : 2;
  p.vec_ok = al16(a.C) && ((a.ldc * esz) % 16 == 0) && ((a.batch_stride_c * esz) % 16 == 0) &&
             ((a.batch2_stride_c * esz) % 16 == 0);
  p.r_vec = a.residual && al16(a.residual) && ((a.ldr * esz) % 16 == 0) && ((a.batch_stride_r * esz) % 16 == 0) &&
            ((a.batch2_stride_r * esz) % 16 == 0);
  p.m_vec = a.relu_mask && al16(a.relu_mask) && ((a.ldm * esz) % 16 == 0) && ((a.batch_stride_m * esz) % 16 == 0) &&
            ((a.batch2_stride_m * esz) % 16 == 0);
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.bias = a.bias;
  p.bias_f32 = (a.bias_dtype == (int)DType::F32);
  p.row_bias = a.row_bias;
  p.a_bcast = a_bcast ? 1 : 0;
  p.bits_out = a.relu_bits_out;
  p.bits_in = a.relu_bits;
  p.ldbits = a.ldbits;
  p.act = a.act;
  p.err = err;
  p.colsum = a.colsum;
  p.tf32 = tf32 ? 1 : 0;
  p.splits = splits;
  p.kb_per_split = (int)(((a.K + bke - 1) / bke + splits - 1) / splits);
  p.split_stride = 0;
  p.sk = sk ? 1 : 0;
  if ((splits > 1 || sk) && red) {
    // Every split's (stream-K unit's) epilogue adds alpha * partial into C
    // with a TMA reduce; C starts from zero (beta = 0) or from its old value
    // (beta = 1).
    p.beta = 0.f;  // the epilogue itself never reads C
    const CUtensorMap tc = make_c_map(p, a.M, a.N, true);
    if (p.tma_c == 2) {
      if (a.beta == 0.f)
        DLVK_CUDA_CHECK(cudaMemset2DAsync(a.C, (size_t)a.ldc * 4, 0, (size_t)a.N * 4, (size_t)a.M, s));
      if (pair && BN == 512) launch_tc_pair<512>(ta, tb, tc, p, max_ctas, s);
    else if (pair) launch_tc_pair<256>(ta, tb, tc, p, max_ctas, s);
      else if (BN == 256) launch_tc<256>(ta, tb, tc, p, max_ctas, s);
      else launch_tc<128>(ta, tb, tc, p, max_ctas, s);
      return;
    }
    // The map was refused: run unsplit.
    p.beta = a.beta;
    splits = 1;
    p.splits = 1;
    p.sk = 0;
    p.kb_per_split = (int)((a.K + bke - 1) / bke);
  }
  if (splits > 1) {
    // Partial accumulators go to the fp32 workspace; the reduce kernel
    // applies alpha/beta/bias/residual/act/mask and writes C.
    const int64_t per = a.M * a.N * a.batch * a.batch2;
    p.C = workspace;
    p.out_f32 = 1;
    p.ldc = a.N;
    p.bsc = a.M * a.N * a.batch2;
    p.bsc2 = a.M * a.N;
    p.split_stride = per;
    p.vec_ok = al16(workspace) && (a.N % 4 == 0);
    p.alpha = 1.f;
    p.beta = 0.f;
    p.bias = nullptr;
    p.row_bias = nullptr;
    p.bits_in = nullptr;
    p.R = nullptr;
    p.Mk = nullptr;
    p.act = ACT_NONE;
    const CUtensorMap tc = make_c_map(p, a.M, a.N);
    if (pair && BN == 512) launch_tc_pair<512>(ta, tb, tc, p, max_ctas, s);
    else if (pair) launch_tc_pair<256>(ta, tb, tc, p, max_ctas, s);
    else if (BN == 256) launch_tc<256>(ta, tb, tc, p, max_ctas, s);
    else launch_tc<128>(ta, tb, tc, p, max_ctas, s);
    const int g = (int)std::min<int64_t>((per + 255) / 256, 148 * 16);
    if (out_dt == DType::F32) splitk_reduce_kernel<float><<<g, 256, 0, s>>>(workspace, splits, per, a);
    else splitk_reduce_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(workspace, splits, per, a);
    DLVK_POST_LAUNCH();
    return;
  }
  const CUtensorMap tc = make_c_map(p, a.M, a.N);
  DLVK_CHECK(!(p.colsum && p.beta == 0.f && !(p.out_f32 && (p.R || p.Mk)) && p.tma_c == 0),
             "gemm_tc: column sums without a staged input need the TMA-store epilogue");
  if (pair && BN == 512) launch_tc_pair<512>(ta, tb, tc, p, max_ctas, s);
  else if (pair) launch_tc_pair<256>(ta, tb, tc, p, max_ctas, s);
  else if (BN == 256) launch_tc<256>(ta, tb, tc, p, max_ctas, s);
  else launch_tc<128>(ta, tb, tc, p, max_ctas, s);
}
}  // namespace

void gemm_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas, float* workspace,
             int64_t workspace_floats) {
  DLVK_CHECK(gemm_tc_supported(a), "gemm_tc: unsupported layout/alignment");
  gemm_tc_impl(out_dt, a, s, err, max_ctas, workspace, workspace_floats, false);
}

bool gemm_tf32_tc_supported(const GemmArgs& a) {
  const bool a_k = (a.sak == 1), a_m = (a.sam == 1) && !a_k;
  const bool b_k = (a.sbk == 1), b_n = (a.sbn == 1) && !b_k;
  if (!(a_k || a_m) || !(b_k || b_n)) return false;
  const int64_t lda = a_k ? a.sam : a.sak;
  const int64_t ldb = b_k ? a.sbn : a.sbk;
  if ((lda * 4) % 16 || (ldb * 4) % 16) return false;
  if (a.batch > 1 && ((a.batch_stride_a * 4) % 16 || (a.batch_stride_b * 4) % 16)) return false;
  if (a.batch2 > 1 && ((a.batch2_stride_a * 4) % 16 || (a.batch2_stride_b * 4) % 16)) return false;
  if (a.batch * a.batch2 * ((a.M + 127) / 128) * ((a.N + 127) / 128) > (1LL << 31) - 1) return false;
  if (!al16(a.A) || !al16(a.B)) return false;
  if (a.M < 1 || a.N < 16 || a.K < 1) return false;
  if (a.M > (1LL << 31) - 1 || a.N > (1LL << 31) - 1 || a.K > (1LL << 31) - 1) return false;
  return true;
}

void gemm_tf32_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas, float* workspace,
                  int64_t workspace_floats) {
  DLVK_CHECK(gemm_tf32_tc_supported(a), "gemm_tf32_tc: unsupported layout/alignment");
  gemm_tc_impl(out_dt, a, s, err, max_ctas, workspace, workspace_floats, true);
}

namespace {
// hi = x rounded to tf32 (10 explicit mantissa bits; the low 13 bits zero),
// lo = x - hi (exact in fp32).  Rounding is to nearest, ties away from zero,
// done with integer arithmetic on the bit pattern; non-finite values pass
// through in hi with lo = 0.
__global__ void tf32_split_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const uint32_t u = __float_as_uint(v);
    float h = v, l = 0.f;
    if ((u & 0x7f800000u) != 0x7f800000u) {
      const uint32_t r = (u + 0x1000u) & 0xffffe000u;  // add half an ulp of tf32, truncate
      h = __uint_as_float(r);
      l = v - h;
    }
    hi[i] = h;
    lo[i] = l;
  }
}
}  // namespace

void tf32_split(const float* x, float* hi, float* lo, int64_t n, cudaStream_t s) {
  if (n <= 0) return;
  const int g = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
  tf32_split_kernel<<<g, 256, 0, s>>>(x, hi, lo, n);
  DLVK_POST_LAUNCH();
}

namespace {
int& pair_flag() {
  static int f = [] {
    const char* e = std::getenv("DLVK_GEMM_PAIR");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return f;
}
}  // namespace

bool gemm_tc_pair_enabled() { return pair_flag() != 0; }

void gemm_tc_set_pair(bool on) { pair_flag() = on ? 1 : 0; }

void gemm_tc_set_wide(int mode) { wide_flag() = mode; }

void gemm_tc_plan(DType out_dt, const GemmArgs& a, int max_ctas, int* bn, int* splits, int* pair) {
  int BN = 256, sp = 1;
  bool pr = false;
  bool sk = false;
  choose_tiling(a, max_ctas > 0 ? max_ctas : sm_count(), BN, sp, pr, split_red_ok(out_dt, a), out_dt == DType::F32,
                false, &sk);
  *bn = BN;
  *splits = sk ? -1 : sp;  // -1: stream-K
  *pair = (pr && max_ctas != 1) ? 1 : 0;
}

int64_t gemm_tc_workspace_floats(const GemmArgs& a, int max_ctas, DType out_dt, bool tf32) {
  if (split_red_ok(out_dt, a) || a.colsum != nullptr) return 0;
  int BN = 256, splits = 1;
  bool pair = false;
  choose_tiling(a, max_ctas > 0 ? max_ctas : sm_count(), BN, splits, pair, false, out_dt == DType::F32, tf32);
  return splits > 1 ? (int64_t)splits * a.M * a.N * a.batch * a.batch2 : 0;
}

}  // namespace dlvk

namespace dlvk {

bool gemm_i8_tc_supported(const void* A, const void* Bt, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return al(A) && al(Bt) && K % 16 == 0 && lda % 16 == 0 && ldb % 16 == 0 && M >= 1 && N >= 16 && K >= 16 &&
         M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31);
}

// int8 x int8 -> int32 on the tensor cores (tcgen05.mma kind::i8), both
// operands K-major (A [M,K], Bt [N,K]), dequantised in the epilogue:
// C = act(acc * row_scale[m] * col_scale[n] + bias[n]).
void gemm_i8_tc(const int8_t* A, const int8_t* Bt, const float* row_scale, const float* col_scale, const float* bias,
                int act, void* C, DType out_dt, int64_t ldc, int64_t M, int64_t N, int64_t K, int64_t lda,
                int64_t ldb, cudaStream_t s, uint32_t* err) {
  DLVK_CHECK(gemm_i8_tc_supported(A, Bt, M, N, K, lda, ldb), "gemm_i8_tc: unsupported shape/alignment");
  {
    thread_local int bound_dev = -1;
    int dev = 0;
    DLVK_CUDA_CHECK(cudaGetDevice(&dev));
    if (bound_dev != dev) {
      DLVK_CUDA_CHECK(cudaSetDevice(dev));
      bound_dev = dev;
    }
  }
  const int BN = N >= 256 ? 256 : 128;
  CUtensorMap ta = make_tmap(A, K, M, 1, 1, lda, lda * M, lda * M, BM, Elem::I8);
  CUtensorMap tb = make_tmap(Bt, K, N, 1, 1, ldb, ldb * N, ldb * N, BN, Elem::I8);
  TcParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = 1;
  p.batch2 = 1;
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)((N + BN - 1) / BN);
  p.C = C;
  p.ldc = ldc;
  p.out_f32 = out_dt == DType::F32;
  const int esz = p.out_f32 ? 4 : 2;
  p.vec_ok = ((reinterpret_cast<uintptr_t>(C) & 15u) == 0) && ((ldc * esz) % 16 == 0);
  p.alpha = 1.f;
  p.bias = bias;
  p.bias_f32 = 1;
  p.act = act;
  p.err = err;
  p.splits = 1;
  p.kb_per_split = (int)((K + 2 * BK - 1) / (2 * BK));
  p.i8 = 1;
  p.row_scale = row_scale;
  p.col_scale = col_scale;
  if (BN == 256) launch_tc<256>(ta, tb, ta, p, 0, s);
  else launch_tc<128>(ta, tb, ta, p, 0, s);
}

}  // namespace dlvk
