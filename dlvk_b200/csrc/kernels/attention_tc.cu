// Fused multi-head attention on the 5th-generation tensor cores (tcgen05),
// forward and backward, for head dim 64 and sequence lengths that are a
// multiple of 128 (non-causal, no mask: the encoder attention of the
// reference's MultiHeadAttentionLayer, include/dlvk/layers/modern_layers.h:
// 75-129; its shader shaders/multi_head_attention.comp:33-114 never
// normalised the softmax).
//
// Q, K and V are read in place from the fused QKV projection output
// [B, S, 3, H, 64] (bf16) through one 2-D TMA map over [B*S, 3*H*64].
//
// Forward (flash_fwd_kernel): persistent CTAs walk (batch, head, 128-query
// tile) items, two at a time (see the kernel).  Warp 0 issues TMA loads (Q
// per stream, K/V in a 5-stage ring), warp 1 issues tcgen05.mma (S = Q K^T
// into a TMEM score buffer per stream; O += P V into a TMEM accumulator,
// with P read from TMEM), and the softmax warps own one query row per
// thread: they load the whole score row from TMEM into registers (releasing
// the score buffer at once), keep the online max / sum in the log2 domain,
// rescale O in TMEM only when a row's max grew by more than 2^8
// (warp-uniform decision, since tcgen05.ld/st are warp-collective), write P
// as bf16 pairs into TMEM for the next MMA, and finally normalise O and
// store it with the row's log-sum-exp (log2 units) for the backward pass.
//
// Backward (flash_bwd_kernel): persistent CTAs walk (batch, head, 128-key
// tile) items with K and V resident.  For each query tile the MMA warp
// computes S^T = K Q^T and dP^T = V dO^T into TMEM; warps 2..9 (two per
// TMEM lane quarter, one key row per thread, half the queries each) rebuild
// P^T = exp2(S^T c - lse) and dS^T = P^T (dP^T - delta) into shared memory;
// the MMA warp then accumulates dV += P^T dO and dK += dS^T Q in TMEM and
// computes dQ = dS K reading the same dS^T tile as an MN-major operand.
// Software pipeline: P^T / dS^T are double-buffered, so the compute warps
// build step g+1's tiles while the tensor cores run step g's gradient MMAs;
// the next query tile's S^T / dP^T are issued as soon as the compute warps
// have read the current ones; dQ alternates between two TMEM buffers whose
// readout happens one step late.  The dQ tile goes through shared memory to
// the global fp32 accumulator with TMA bulk reduce-add; dK / dV are written
// to the fused gradient buffer [B, S, 3, H, 64] when the key tile is done.
//
// Every mbarrier wait is bounded (mbar_wait: error word + early exit).
#include <cuda.h>

#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/sm100.h"
#include "dlvk/tmap.h"

namespace dlvk {
namespace {
using namespace sm100;

constexpr int FT = 128;                  // query / key tile
constexpr int FD = 64;                   // head dim
constexpr int TILE = FT * FD * 2;        // one bf16 [128 x 64] tile, 16 KB

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk `c` (8 bf16, c in 0..15) of row `r` in a
// [128 x 128] bf16 K-major operand stored as two 128-byte-swizzled
// [128 x 64] sub-tiles (the layout TMA SWIZZLE_128B produces).
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 3) * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// 2^x with the hardware approximation (ex2.approx.ftz: flushes denormal
// results to zero, which bf16 probabilities cannot represent anyway).
__device__ __forceinline__ float hw_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^(-x): the negation folds into the exponential's operand.
__device__ __forceinline__ float hw_exp2_neg(float x) {
  float y;
  asm("{\n\t.reg .f32 t;\n\tneg.f32 t, %1;\n\tex2.approx.ftz.f32 %0, t;\n\t}" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float2 f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }

// Bounded wait whose outcome is the same in every lane of the warp (the
// warp-collective tcgen05.ld / st that follow need all 32 lanes).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

struct FwdP {
  __nv_bfloat16* out;
  float* lse;
  int B, S, H, E;
  float c;  // softmax scale * log2(e)
  uint32_t* err;
};

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16: A is read from tensor
// memory (lane = row, two bf16 per 32-bit column, K-major), B from shared
// memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Two softmax warpgroups ("streams" 0 and 1) work on independent items in
// ping-pong: CTA c gives items c, c + 2g, ... to stream 0 and c + g,
// c + 3g, ... to stream 1 (g = grid size).  Each stream has its own TMEM
// score buffer S, probability tile P and output accumulator O, and its own
// Q tile in shared memory; the K / V ring, the TMA producer warp and the MMA
// warp are shared.  While one stream normalises and stores its finished
// item, or waits for its next scores, the other keeps the exponential unit
// busy.
//
// TMEM (512 columns): S0 0..127, S1 128..255, O0 256..319, O1 320..383,
// P0 384..447, P1 448..511 (P as bf16 pairs: 128 keys in 64 columns).  The
// PV product reads P straight from tensor memory.
// Shared memory: Q x2 | (K, V) x FWD_KV_STAGES | barriers.
constexpr int FWD_KV_STAGES = 5;
constexpr int FWD_THREADS = 64 + 2 * 128;
constexpr int FWD_SMEM = 2 * TILE + FWD_KV_STAGES * 2 * TILE + 256 + 1024;

__global__ void __launch_bounds__(FWD_THREADS, 1) flash_fwd_kernel(const __grid_constant__ CUtensorMap tm, FwdP p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                   // stream t: sQ + t * TILE
  uint8_t* sKV = smem + 2 * TILE;                       // stage k: K at k * 2 * TILE, V at + TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + FWD_KV_STAGES * 2 * TILE);
  uint64_t* q_full = bars;                              // [2] per stream
  uint64_t* q_empty = bars + 2;                         // [2]
  uint64_t* kv_full = bars + 4;                         // [FWD_KV_STAGES]
  uint64_t* kv_empty = bars + 4 + FWD_KV_STAGES;        // [FWD_KV_STAGES]
  uint64_t* s_full = bars + 4 + 2 * FWD_KV_STAGES;      // [2]
  uint64_t* s_empty = s_full + 2;                       // [2], 4 warp arrivals
  uint64_t* p_full = s_full + 4;                        // [2], 4 warp arrivals
  uint64_t* pv_done = s_full + 6;                       // [2]
  uint64_t* o_empty = s_full + 8;                       // [2], 4 warp arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = p.S / FT;
  const int items = p.B * p.H * nt;
  const int g = (int)gridDim.x;
  // Item of stream t in round r of this CTA (>= items: none).
  auto item_of = [&](int r, int t) { return (int)blockIdx.x + (2 * r + t) * g; };

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&s_empty[t], 4);
      mbar_init(&p_full[t], 4);
      mbar_init(&pv_done[t], 1);
      mbar_init(&o_empty[t], 4);
    }
    for (int i = 0; i < FWD_KV_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm);
      int kvs = 0;
      uint32_t kvph = 0;
      bool ok = true;
      // Loads in the MMA warp's consumption order: round r, tile j, stream 0 then 1.
      for (int r = 0; ok && item_of(r, 0) < items; ++r) {
        for (int j = 0; ok && j < nt; ++j) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int item = item_of(r, t);
            if (item >= items) continue;
            const int qt = item % nt, bh = item / nt, h = bh % p.H, b = bh / p.H;
            if (j == 0) {
              if (!mbar_wait(&q_empty[t], (r & 1) ^ 1u, p.err)) { ok = false; break; }
              mbar_arrive_expect_tx(&q_full[t], TILE);
              tma_load_2d(sQ + t * TILE, &tm, &q_full[t], h * FD, b * p.S + qt * FT);
            }
            if (!mbar_wait(&kv_empty[kvs], kvph ^ 1u, p.err)) { ok = false; break; }
            uint8_t* k = sKV + kvs * 2 * TILE;
            mbar_arrive_expect_tx(&kv_full[kvs], 2 * TILE);
            tma_load_2d(k, &tm, &kv_full[kvs], p.E + h * FD, b * p.S + j * FT);
            tma_load_2d(k + TILE, &tm, &kv_full[kvs], 2 * p.E + h * FD, b * p.S + j * FT);
            if (++kvs == FWD_KV_STAGES) {
              kvs = 0;
              kvph ^= 1u;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = make_idesc(1, 1, 1, false, false, 128, 128);
      const uint32_t id_o = make_idesc(1, 1, 1, false, true, 128, 64);
      int kvs = 0;
      uint32_t kvph = 0;
      // Per-stream MMA state (scalars, not arrays indexed by the stream, so
      // it stays in registers).
      struct St {
        uint32_t sph, pph, oph;
        int prev;  // K/V stage of the stream's previous tile (its PV is pending)
        int cur;   // K/V stage of the tile whose S was just issued
      };
      St st0{0, 0, 0, 0, 0}, st1{0, 0, 0, 0, 0};
      bool ok = true;
      // Round j: both streams' S for tile j, then both streams' PV for tile
      // j - 1, so neither stream's scores wait behind the other's softmax.
      auto stepS = [&](int r, int j, int t, St& st) {
        if (item_of(r, t) >= items || j >= nt) return true;
        const uint32_t tS = tbase + (uint32_t)(t * 128);
        if (j == 0 && !mbar_wait(&q_full[t], r & 1, p.err)) return false;
        if (!mbar_wait(&kv_full[kvs], kvph, p.err) || !mbar_wait(&s_empty[t], st.sph ^ 1u, p.err)) return false;
        st.sph ^= 1u;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + t * TILE), ka = smem_u32(sKV + kvs * 2 * TILE);
#pragma unroll
        for (int k = 0; k < FD / 16; ++k)
          mma_f16(tS, make_sw128_desc(qa + k * 32, 16, 1024), make_sw128_desc(ka + k * 32, 16, 1024), id_s,
                  k ? 1u : 0u);
        mma_commit(&s_full[t]);
        if (j == nt - 1) mma_commit(&q_empty[t]);
        st.cur = kvs;
        if (++kvs == FWD_KV_STAGES) {
          kvs = 0;
          kvph ^= 1u;
        }
        return true;
      };
      auto stepPV = [&](int r, int j, int t, St& st) {
        if (item_of(r, t) >= items || j == 0) return true;
        const uint32_t tO = tbase + 256u + (uint32_t)(t * 64), tP = tbase + 384u + (uint32_t)(t * 64);
        if (j == 1) {
          if (!mbar_wait(&o_empty[t], st.oph ^ 1u, p.err)) return false;
          st.oph ^= 1u;
        }
        if (!mbar_wait(&p_full[t], st.pph, p.err)) return false;
        st.pph ^= 1u;
        tc_fence_after();
        const uint32_t va = smem_u32(sKV + st.prev * 2 * TILE + TILE);
        // O += P V: A = P from TMEM (16 keys = 8 columns per MMA), B = V
        // MN-major [keys x d].
#pragma unroll
        for (int k = 0; k < FT / 16; ++k)
          mma_f16_ts(tO, tP + (uint32_t)(k * 8), make_sw128_desc(va + k * 2048, 16384, 1024), id_o,
                     (j > 1 || k > 0) ? 1u : 0u);
        mma_commit(&kv_empty[st.prev]);
        mma_commit(&pv_done[t]);
        return true;
      };
      for (int r = 0; ok && item_of(r, 0) < items; ++r)
        for (int j = 0; ok && j <= nt; ++j) {
          ok = stepS(r, j, 0, st0) && stepS(r, j, 1, st1) && stepPV(r, j, 0, st0) && stepPV(r, j, 1, st1);
          st0.prev = st0.cur;
          st1.prev = st1.cur;
        }
    }
  } else {
    // Softmax warps: stream t = (warp - 2) / 4; warp w reads TMEM lanes
    // 32 * (w % 4) .. + 31 (row = query).
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tbase + lane_off + (uint32_t)(t * 128), tO = tbase + lane_off + 256u + (uint32_t)(t * 64);
    const uint32_t tP = tbase + lane_off + 384u + (uint32_t)(t * 64);
    uint32_t sph = 0, pvph = 0;
    for (int r = 0;; ++r) {
      const int item = item_of(r, t);
      if (item >= items) break;
      const int qt = item % nt, bh = item / nt, h = bh % p.H, b = bh / p.H;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        if (!warp_wait(&s_full[t], sph, p.err)) { ok = false; break; }
        sph ^= 1u;
        tc_fence_after();
        // The whole score row (128 keys) in registers, so the score buffer
        // is released right away for the stream's next tile.
        uint32_t sc[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + (uint32_t)(c * 32), sc[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[t]);
        float mp[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mp[k] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(sc[c][i]));
        float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
        mx *= p.c;
        const bool need = mx > m + 8.f;  // lazy rescale: keep the old reference max while it is within 2^8
        const float m_new = need ? mx : m;
        const float alpha = need ? hw_exp2(m - m_new) : 1.f;
        if (j > 0) {
          // The previous tile's PV must be done before P is rewritten or O
          // rescaled.
          if (!warp_wait(&pv_done[t], pvph, p.err)) { ok = false; break; }
          pvph ^= 1u;
          tc_fence_after();
        }
        // Exponentials straight to P (bf16 pairs in TMEM); the row sum uses
        // the fp32 values.  (Packed fp32 pairs measured the same here and
        // spill under the 168-register cap.)
        float sp8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) sp8[k] = 0.f;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const int c = 2 * hf + (i >> 5);
            const float e0 = hw_exp2(fmaf(__uint_as_float(sc[c][i & 31]), p.c, -m_new));
            const float e1 = hw_exp2(fmaf(__uint_as_float(sc[c][(i & 31) + 1]), p.c, -m_new));
            sp8[i & 7] += e0;
            sp8[(i + 1) & 7] += e1;
            pk[i >> 1] = pack2(e0, e1);
          }
          tmem_st32(tP + (uint32_t)(hf * 32), pk);
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + (uint32_t)(c * 32), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + (uint32_t)(c * 32), o);
          }
        }
        tmem_st_wait();
        l = l * alpha + (((sp8[0] + sp8[1]) + (sp8[2] + sp8[3])) + ((sp8[4] + sp8[5]) + (sp8[6] + sp8[7])));
        m = m_new;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      if (!warp_wait(&pv_done[t], pvph, p.err)) break;
      pvph ^= 1u;
      tc_fence_after();
      // O row in two 32-column halves: normalise and store each (a thread
      // writes its row's 128 bytes as eight 16-byte stores).
      const float inv = 1.f / l;
      const int64_t grow = (int64_t)b * p.S + (int64_t)qt * FT + row;
      uint4* dst = reinterpret_cast<uint4*>(p.out + grow * p.E + h * FD);
      uint32_t o[2][32];
      tmem_ld32(tO, o[0]);
      tmem_ld32(tO + 32u, o[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[t]);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t* src = &o[hf][c * 8];
          uint4 v;
          v.x = pack2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          v.y = pack2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          v.z = pack2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          v.w = pack2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
          dst[hf * 4 + c] = v;
        }
      }
      p.lse[((int64_t)b * p.H + h) * p.S + (int64_t)qt * FT + row] = m + log2f(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  pdl_trigger();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------- backward
struct BwdP {
  const float* lse;    // [B, H, S] log2 units
  const float* delta;  // [B, H, S] -rowsum(dO * O)
  __nv_bfloat16* dqkv; // [B, S, 3E]
  int B, S, H, E;
  float c;             // scale * log2(e)
  float scale;
  uint32_t* err;
};

// Shared memory: K | V | (Q, dO) x2 | P^T x2 (32 KB each) | dS^T x2 |
// (lse, delta) x2 | barriers.  The producer copies each query tile's lse and
// delta (128 floats each) into the stage of its Q / dO tiles, in the same
// transaction.  P^T and dS^T are double-buffered (step g uses buffer
// g & 1) so that the compute warps build step g+1's tiles while the tensor
// cores run step g's gradient MMAs.  Step g's dQ tile is staged for its TMA
// reduce-add in P^T buffer g & 1, which is free from the end of step g's
// gradient MMAs until step g+2 writes its P^T there.
constexpr int BWD_SMEM_USED = 14 * TILE + 4 * 128 * 4 + 256;
constexpr int BWD_SMEM = 227 * 1024;  // the opt-in maximum; the kernel checks that the base alignment fits
static_assert(BWD_SMEM_USED <= BWD_SMEM, "backward shared memory");

__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completion counted on `bar` in bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr int BWD_COMPUTE_WARPS = 8;  // two per TMEM lane quarter
constexpr int BWD_THREADS = 64 + 32 * BWD_COMPUTE_WARPS;

__global__ void __launch_bounds__(BWD_THREADS, 1) flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                                                           const __grid_constant__ CUtensorMap tm_do,
                                                           const __grid_constant__ CUtensorMap tm_dq, BwdP p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // The layout needs all but 768 bytes of the allocation: a dynamic
  // shared-memory base further than that from a 1024-byte boundary cannot
  // hold it (the same decision in every thread, before any barrier).
  if ((int)(smem - smem_raw) + BWD_SMEM_USED > BWD_SMEM) {
    if (threadIdx.x == 0) atomicCAS(p.err, 0u, (uint32_t)DLVK_ERR_BAD_ARG);
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = smem + TILE;
  uint8_t* sQD = smem + 2 * TILE;            // stage s: Q at s*2*TILE, dO at +TILE
  uint8_t* sPT = smem + 6 * TILE;            // buffer u at u*2*TILE (32 KB each)
  uint8_t* sDS = smem + 10 * TILE;           // buffer u at u*2*TILE
  float* sLD = reinterpret_cast<float*>(smem + 14 * TILE);    // stage s: lse at s*256, delta at s*256 + 128
  uint64_t* bars = reinterpret_cast<uint64_t*>(sLD + 512);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + 1;
  uint64_t* qd_full = bars + 2;   // 2
  uint64_t* qd_empty = bars + 4;  // 2
  uint64_t* st_full = bars + 6;
  uint64_t* ds_full = bars + 7;   // 2: P^T / dS^T buffer u written
  uint64_t* dq_full = bars + 9;   // 2: gradient MMAs of a step using dQ TMEM buffer u complete
  uint64_t* dq_free = bars + 11;  // 2: dQ TMEM buffer u read out
  uint64_t* kv_done = bars + 13;  // dK, dV accumulated for the item
  uint64_t* kv_read = bars + 14;  // dK, dV read out of TMEM
  uint64_t* st_free = bars + 15;  // S^T / dP^T read out of TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = p.S / FT;
  const int items = p.B * p.H * nt;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&ds_full[i], BWD_COMPUTE_WARPS);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], BWD_COMPUTE_WARPS);
    }
    mbar_init(st_full, 1);
    mbar_init(kv_done, 1);
    mbar_init(kv_read, BWD_COMPUTE_WARPS);
    mbar_init(st_free, BWD_COMPUTE_WARPS);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // TMEM: S^T 0..127, dP^T 128..255, dV 256..319, dK 320..383, dQ of step g at 384 + 64 * (g & 1)
  const uint32_t tbase = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_qkv);
      prefetch_tmap(&tm_do);
      int it = 0, qs = 0;
      uint32_t qph = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++it) {
        const int kt = item % nt, bh = item / nt, h = bh % p.H, b = bh / p.H;
        if (!mbar_wait(kv_empty, (it & 1) ^ 1u, p.err)) break;
        mbar_arrive_expect_tx(kv_full, 2 * TILE);
        tma_load_2d(sK, &tm_qkv, kv_full, p.E + h * FD, b * p.S + kt * FT);
        tma_load_2d(sV, &tm_qkv, kv_full, 2 * p.E + h * FD, b * p.S + kt * FT);
        for (int i = 0; i < nt; ++i) {
          if (!mbar_wait(&qd_empty[qs], qph ^ 1u, p.err)) { ok = false; break; }
          uint8_t* d = sQD + qs * 2 * TILE;
          const int64_t lo = ((int64_t)b * p.H + h) * p.S + (int64_t)i * FT;
          mbar_arrive_expect_tx(&qd_full[qs], 2 * TILE + 2 * FT * 4);
          tma_load_2d(d, &tm_qkv, &qd_full[qs], h * FD, b * p.S + i * FT);
          tma_load_2d(d + TILE, &tm_do, &qd_full[qs], h * FD, b * p.S + i * FT);
          bulk_load(sLD + qs * 256, p.lse + lo, FT * 4, &qd_full[qs]);
          bulk_load(sLD + qs * 256 + 128, p.delta + lo, FT * 4, &qd_full[qs]);
          if (++qs == 2) {
            qs = 0;
            qph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_st = make_idesc(1, 1, 1, false, false, 128, 128);  // S^T, dP^T: K-major A and B
      const uint32_t id_kv = make_idesc(1, 1, 1, false, true, 128, 64);    // dV, dK: K-major A, MN-major B
      const uint32_t id_q = make_idesc(1, 1, 1, true, true, 128, 64);      // dQ: MN-major A and B
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      // Steps are numbered g across items; step g uses Q / dO stage, P^T /
      // dS^T buffer and dQ TMEM buffer g & 1.  Step g+1's S^T / dP^T go out
      // as soon as the compute warps have read step g's (st_free), ahead of
      // step g's gradient MMAs.
      int64_t g = 0;
      uint32_t stfph = 0;
      bool ok = true;
      auto issue_scores = [&](int64_t gs) -> bool {
        const int st = (int)(gs & 1);
        if (!mbar_wait(&qd_full[st], (uint32_t)((gs >> 1) & 1), p.err)) return false;
        if (gs > 0) {
          if (!mbar_wait(st_free, stfph, p.err)) return false;  // step gs-1's scores read out of TMEM
          stfph ^= 1u;
        }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQD + st * 2 * TILE), doa = qa + TILE;
#pragma unroll
        for (int k = 0; k < FD / 16; ++k) {
          mma_f16(tbase, make_sw128_desc(ka + k * 32, 16, 1024), make_sw128_desc(qa + k * 32, 16, 1024), id_st,
                  k ? 1u : 0u);
          mma_f16(tbase + 128, make_sw128_desc(va + k * 32, 16, 1024), make_sw128_desc(doa + k * 32, 16, 1024),
                  id_st, k ? 1u : 0u);
        }
        mma_commit(st_full);
        return true;
      };
      for (int item = blockIdx.x, it = 0; item < items && ok; item += gridDim.x, ++it) {
        if (!mbar_wait(kv_full, it & 1, p.err)) break;
        if (!issue_scores(g)) break;
        for (int i = 0; i < nt; ++i, ++g) {
          const int cur = (int)(g & 1);
          const uint32_t par = (uint32_t)((g >> 1) & 1);
          if (i + 1 < nt && !issue_scores(g + 1)) { ok = false; break; }
          if (!mbar_wait(&ds_full[cur], par, p.err)) { ok = false; break; }
          if (i == 0 && !mbar_wait(kv_read, (it & 1) ^ 1u, p.err)) { ok = false; break; }  // previous dK / dV read
          // dQ buffer g & 1 was read out two steps ago
          if (!mbar_wait(&dq_free[cur], par ^ 1u, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tdq = tbase + 384 + 64 * cur;
          const uint32_t qa = smem_u32(sQD + cur * 2 * TILE), doa = qa + TILE;
          const uint32_t pta = smem_u32(sPT + cur * 2 * TILE), dsa = smem_u32(sDS + cur * 2 * TILE);
#pragma unroll
          for (int k = 0; k < FT / 16; ++k) {
            const uint32_t koff = (uint32_t)((k >> 2) * 16384 + (k & 3) * 32);
            // dV += P^T dO, dK += dS^T Q: A K-major [keys x queries], B = dO / Q as MN-major [queries x d]
            mma_f16(tbase + 256, make_sw128_desc(pta + koff, 16, 1024), make_sw128_desc(doa + k * 2048, 16384, 1024),
                    id_kv, (i > 0 || k > 0) ? 1u : 0u);
            mma_f16(tbase + 320, make_sw128_desc(dsa + koff, 16, 1024), make_sw128_desc(qa + k * 2048, 16384, 1024),
                    id_kv, (i > 0 || k > 0) ? 1u : 0u);
            // dQ = dS K: A = dS^T tile read MN-major (M = queries in 64-wide chunks 16 KB apart), B = K MN-major
            mma_f16(tdq, make_sw128_desc(dsa + k * 2048, 16384, 1024),
                    make_sw128_desc(ka + k * 2048, 16384, 1024), id_q, k > 0 ? 1u : 0u);
          }
          mma_commit(&dq_full[cur]);
          mma_commit(&qd_empty[cur]);
        }
        if (!ok) break;
        mma_commit(kv_empty);
        mma_commit(kv_done);
      }
    }
  } else {
    // Compute warps 2..9: warp w reads TMEM lanes 32*(w%4).. (row = key for
    // S^T, dP^T, dK, dV; query for dQ); `hf` selects which half of the
    // columns (queries of S^T / dP^T, dQ columns, dV vs dK) it handles.
    const int quarter = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t stph = 0;
    int it = 0;
    int64_t g = 0;
    bool ok = true;
    // The dQ tile of step g leaves TMEM during step g+1, after that step's
    // P^T / dS^T tiles are written: it sits in one of two TMEM buffers, so
    // the gradient MMAs of step g+1 need not wait for it.  dq_x / dq_y are
    // its coordinates in dQ.
    bool dq_pending = false;
    int dq_x = 0, dq_y = 0;
    // Box of this warp inside a P^T buffer: the same 4 KB this warp writes
    // its P^T rows into (rows 32 * quarter.., 16-byte chunks 8 * hf..).
    const int box_off = hf * 16384 + quarter * 4096;
    // Step gd's gradient MMAs complete -> dQ from TMEM -> registers -> this
    // warp's 32 x 32 fp32 box (swizzled as the map expects) in P^T buffer
    // gd & 1 -> TMA reduce-add issued by the warp's lane 0.
    auto reduce_dq = [&](int64_t gd) -> bool {
      const int u = (int)(gd & 1);
      if (!warp_wait(&dq_full[u], (uint32_t)((gd >> 1) & 1), p.err)) return false;
      tc_fence_after();
      uint32_t qv[32];
      tmem_ld32(tbase + lane_off + 384u + (uint32_t)(64 * u + hf * 32), qv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[u]);
      uint8_t* base = sPT + u * 2 * TILE + box_off + lane * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v = make_uint4(qv[c * 4], qv[c * 4 + 1], qv[c * 4 + 2], qv[c * 4 + 3]);
        *reinterpret_cast<uint4*>(base + ((c ^ (lane & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tm_dq, sPT + u * 2 * TILE + box_off, dq_x + hf * 32, dq_y + quarter * 32);
        bulk_commit();
      }
      return true;
    };
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++it) {
      const int kt = item % nt, bh = item / nt, h = bh % p.H, b = bh / p.H;
      for (int i = 0; i < nt; ++i, ++g) {
        const int u = (int)(g & 1);
        if (!warp_wait(st_full, stph, p.err)) { ok = false; break; }
        stph ^= 1u;
        // this step's lse / delta came with its Q / dO tiles (complete: the
        // scores just computed read those tiles)
        if (!warp_wait(&qd_full[u], (uint32_t)((g >> 1) & 1), p.err)) { ok = false; break; }
        tc_fence_after();
        // All of this warp's scores at once (64 queries of S^T and dP^T), so
        // the score buffer is released before any arithmetic.
        uint32_t s[2][32], dp[2][32];
        tmem_ld32(tbase + lane_off + (uint32_t)(hf * 64), s[0]);
        tmem_ld32(tbase + lane_off + (uint32_t)(hf * 64 + 32), s[1]);
        tmem_ld32(tbase + lane_off + 128u + (uint32_t)(hf * 64), dp[0]);
        tmem_ld32(tbase + lane_off + 128u + (uint32_t)(hf * 64 + 32), dp[1]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_free);  // the next step's S^T / dP^T may overwrite them
        const float* L = sLD + u * 256 + hf * 64;
        const float* Dl = L + 128;  // -delta
        const float2 nc2 = make_float2(-p.c, -p.c);
        // Buffer u was last read by step g-2's gradient MMAs (complete: its
        // dQ was reduced during step g-1) and by the TMA reduce of step g-2's
        // dQ box, which must have finished reading it.
        uint8_t* const PT = sPT + u * 2 * TILE;
        uint8_t* const DS = sDS + u * 2 * TILE;
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {  // 8 queries per 16-byte chunk
          // per-query lse / -delta: 16-byte broadcast loads
          const float4 l0 = *reinterpret_cast<const float4*>(L + c8 * 8);
          const float4 l1 = *reinterpret_cast<const float4*>(L + c8 * 8 + 4);
          const float4 d0 = *reinterpret_cast<const float4*>(Dl + c8 * 8);
          const float4 d1 = *reinterpret_cast<const float4*>(Dl + c8 * 8 + 4);
          const float2 lv[4] = {make_float2(l0.x, l0.y), make_float2(l0.z, l0.w), make_float2(l1.x, l1.y),
                                make_float2(l1.z, l1.w)};
          const float2 nd[4] = {make_float2(d0.x, d0.y), make_float2(d0.z, d0.w), make_float2(d1.x, d1.y),
                                make_float2(d1.z, d1.w)};
          uint32_t pk[4], dk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int e = c8 * 8 + 2 * j;
            // p = 2^(S c - lse), dS = p (dP - delta), in packed fp32 pairs
            const float2 x = __ffma2_rn(f2(s[e >> 5][e & 31], s[e >> 5][(e + 1) & 31]), nc2, lv[j]);
            const float2 pp = make_float2(hw_exp2_neg(x.x), hw_exp2_neg(x.y));
            const float2 ds = __fmul2_rn(pp, __fadd2_rn(f2(dp[e >> 5][e & 31], dp[e >> 5][(e + 1) & 31]), nd[j]));
            pk[j] = pack2(pp.x, pp.y);
            dk[j] = pack2(ds.x, ds.y);
          }
          const int ch = hf * 8 + c8;
          *reinterpret_cast<uint4*>(PT + sw_off(row, ch)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(DS + sw_off(row, ch)) = make_uint4(dk[0], dk[1], dk[2], dk[3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ds_full[u]);
        if (dq_pending && !reduce_dq(g - 1)) { ok = false; break; }
        dq_pending = true;
        dq_x = h * FD;
        dq_y = b * p.S + i * FT;
      }
      if (!ok) break;
      // dV (hf = 0) or dK (hf = 1, scaled) of this key tile -> the fused gradient buffer.
      if (!warp_wait(kv_done, it & 1, p.err)) break;
      tc_fence_after();
      const int64_t grow = (int64_t)b * p.S + (int64_t)kt * FT + row;
      {
        uint32_t a0[32], a1[32];
        tmem_ld32(tbase + lane_off + 256u + (uint32_t)(hf * 64), a0);
        tmem_ld32(tbase + lane_off + 288u + (uint32_t)(hf * 64), a1);
        tmem_ld_wait();
        const float sc = hf ? p.scale : 1.f;
        uint4* dst = reinterpret_cast<uint4*>(p.dqkv + grow * 3 * p.E + (hf ? p.E : 2 * p.E) + h * FD);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* sv = c < 4 ? &a0[c * 8] : &a1[(c - 4) * 8];
          uint4 v;
          v.x = pack2(__uint_as_float(sv[0]) * sc, __uint_as_float(sv[1]) * sc);
          v.y = pack2(__uint_as_float(sv[2]) * sc, __uint_as_float(sv[3]) * sc);
          v.z = pack2(__uint_as_float(sv[4]) * sc, __uint_as_float(sv[5]) * sc);
          v.w = pack2(__uint_as_float(sv[6]) * sc, __uint_as_float(sv[7]) * sc);
          dst[c] = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_read);
    }
    if (ok && dq_pending) reduce_dq(g - 1);
    if (lane == 0) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  pdl_trigger();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// delta[b, h, q] = -sum_d dO[b, q, h, d] * O[b, q, h, d] (stored negated:
// the backward kernel adds it to dP), and the row's 64
// entries of the fp32 dQ accumulator cleared (no separate memset): eight lanes per
// (b, q, h) row of 64, one 16-byte vector of each operand per lane, reduced
// with three shuffles.  A warp reads four consecutive rows (512 contiguous
// bytes per operand per load instruction).
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  float* __restrict__ delta, int B, int S, int H, float* __restrict__ dq_zero) {
  pdl_wait();
  const int64_t total = (int64_t)B * S * H * 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // Warp-uniform trip count: lanes past the end compute zeros and store nothing.
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base < total; base += stride) {
    const int64_t t = base + (threadIdx.x & 31);
    const bool on = t < total;
    const int64_t w = t >> 3;
    float acc = 0.f;
    if (on) {
      const uint4 av = reinterpret_cast<const uint4*>(o + w * FD)[t & 7];
      const uint4 dv = reinterpret_cast<const uint4*>(dout + w * FD)[t & 7];
      const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&av);
      const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&dv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 xf = __bfloat1622float2(x[k]), yf = __bfloat1622float2(y[k]);
        acc = fmaf(xf.x, yf.x, fmaf(xf.y, yf.y, acc));
      }
    }
    if (on) {
      // the same row of the fp32 dQ accumulator [B*S, H*64] starts at zero
      float4* z = reinterpret_cast<float4*>(dq_zero + w * FD) + (t & 7) * 2;
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (on && (t & 7) == 0) {
      const int h = (int)(w % H);
      const int64_t bq = w / H;
      const int q = (int)(bq % S), b = (int)(bq / S);
      delta[((int64_t)b * H + h) * S + q] = -acc;
    }
  }
}

// dqkv[:, :, 0] = bf16(dq_acc * scale)
__global__ void attn_dq_finish_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv, int64_t rows,
                                      int E, float scale) {
  pdl_wait();
  const int64_t n4 = rows * E / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(acc)[i];
    const int64_t e = i * 4;
    const int64_t r = e / E, c = e % E;
    uint2 o;
    o.x = pack2(v.x * scale, v.y * scale);
    o.y = pack2(v.z * scale, v.w * scale);
    *reinterpret_cast<uint2*>(dqkv + r * 3 * E + c) = o;
  }
}

}  // namespace

bool flash_attention_supported(int64_t B, int64_t S, int64_t H, int64_t D, const void* qkv) {
  return D == FD && S % FT == 0 && S > 0 && B > 0 && H > 0 && (reinterpret_cast<uintptr_t>(qkv) & 15u) == 0 &&
         B * S < (1LL << 31) && 3 * H * D < (1LL << 31);
}

void flash_attention_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int B, int S, int H, float scale,
                         cudaStream_t s, uint32_t* err, int max_ctas) {
  DLVK_CHECK(flash_attention_supported(B, S, H, FD, qkv), "flash_attention_fwd: unsupported shape");
  tmap::bind_context();
  const int E = H * FD;
  CUtensorMap tm = tmap::bf16_2d_sw128(qkv, (uint64_t)3 * E, (uint64_t)B * S, (uint64_t)3 * E, FT);
  FwdP p{out, lse, B, S, H, E, scale * 1.4426950408889634f, err};
  auto kern = flash_fwd_kernel;
  const int adev = current_device_slot();
  static bool attr[kMaxDevices] = {};  // per device: the attribute belongs to each device's context
  if (!attr[adev]) {
    DLVK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM));
    attr[adev] = true;
  }
  const int items = B * H * (S / FT);
  int grid = std::min(items, max_ctas > 0 ? max_ctas : tmap::sm_count());
  launch_pdl(kern, dim3(grid), dim3(FWD_THREADS), FWD_SMEM, s, tm, p);
  DLVK_POST_LAUNCH();
}

void flash_attention_bwd(const __nv_bfloat16* qkv, const __nv_bfloat16* out, const __nv_bfloat16* dout,
                         const float* lse, float* delta, float* dq_acc, __nv_bfloat16* dqkv, int B, int S, int H,
                         float scale, cudaStream_t s, uint32_t* err, int max_ctas) {
  DLVK_CHECK(flash_attention_supported(B, S, H, FD, qkv), "flash_attention_bwd: unsupported shape");
  // lse and delta rows are bulk-copied into shared memory (16-byte aligned)
  DLVK_CHECK((reinterpret_cast<uintptr_t>(lse) & 15u) == 0 && (reinterpret_cast<uintptr_t>(delta) & 15u) == 0,
             "flash_attention_bwd: lse and delta must be 16-byte aligned");
  tmap::bind_context();
  const int E = H * FD;
  const int64_t rows = (int64_t)B * S;
  {
    const int64_t n = rows * H * 8;
    launch_pdl(attn_delta_kernel, dim3((unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)tmap::sm_count() * 16)),
               dim3(256), 0, s, out, dout, delta, B, S, H, dq_acc);
    DLVK_POST_LAUNCH();
  }
  CUtensorMap tq = tmap::bf16_2d_sw128(qkv, (uint64_t)3 * E, (uint64_t)rows, (uint64_t)3 * E, FT);
  CUtensorMap td = tmap::bf16_2d_sw128(dout, (uint64_t)E, (uint64_t)rows, (uint64_t)E, FT);
  CUtensorMap tdq;
  {
    cuuint64_t dims[2] = {(cuuint64_t)E, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)E * 4};
    cuuint32_t box[2] = {32u, 32u};  // one compute warp's 32 queries x 32 columns
    cuuint32_t estr[2] = {1, 1};
    CUresult r = tmap::encode_fn()(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc, dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("dlvk: dq tensor map failed (" + std::to_string((int)r) + ")");
  }
  BwdP p{lse, delta, dqkv, B, S, H, E, scale * 1.4426950408889634f, scale, err};
  const int adev = current_device_slot();
  static bool attr[kMaxDevices] = {};  // per device: the attribute belongs to each device's context
  if (!attr[adev]) {
    DLVK_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
    attr[adev] = true;
  }
  const int items = B * H * (S / FT);
  const int grid = std::min(items, max_ctas > 0 ? max_ctas : tmap::sm_count());
  launch_pdl(flash_bwd_kernel, dim3(grid), dim3(BWD_THREADS), BWD_SMEM, s, tq, td, tdq, p);
  DLVK_POST_LAUNCH();
  const int64_t n4 = rows * E / 4;
  launch_pdl(attn_dq_finish_kernel, dim3((unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 16)), dim3(256), 0, s,
             (const float*)dq_acc, dqkv, rows, E, scale);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
