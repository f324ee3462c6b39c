// Tensor-core GEMM for sm_100a: TMA -> shared-memory ring -> tcgen05.mma ->
// TMEM accumulators -> fused epilogue.  Replaces the reference's
// matrix_multiply.comp / batch_matrix_multiply.comp (shaders/, dispatched from
// src/tensor/tensor_ops.cpp:187-298) for Dense forward/backward, attention
// projections and the batched attention products.
//
// Design:
//  * persistent kernel, one CTA per SM, 192 threads = 6 warps:
//      warp 0      TMA producer (one lane) over a STAGES-deep smem ring
//      warp 1      TMEM allocator + MMA issuer (one lane)
//      warps 2..5  epilogue: tcgen05.ld 32x32b -> alpha/beta/bias/act -> global
//  * tile 128 x BN x 64 (BN = 256 or 128), UMMA 128 x BN x 16 (kind::f16, bf16
//    in, f32 accumulate), two TMEM accumulator buffers so the epilogue of tile
//    i overlaps the main loop of tile i+1.
//  * A may be K-major ([M,K] row-major) or M-major ([K,M] row-major); B may be
//    K-major ([N,K]) or N-major ([K,N]).  Both are expressed through the TMA
//    box shape and the UMMA descriptor major-ness, so no transpose kernels are
//    ever needed for X*W, dY*W^T or X^T*dY.
//  * TMA loads are plain (no cluster multicast).
//  * every mbarrier wait is bounded (2 s) and reports through `err`.
#include <cuda.h>
#include <cudaTypedefs.h>
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
};

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_BYTES = 4 * 32 * 33 * 4;  // per-warp 32x33 fp32 staging
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + EPI_BYTES;
};

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

__device__ __forceinline__ float act_apply(int act, float v) {
  if (act == ACT_RELU) return fmaxf(v, 0.f);
  if (act == ACT_GELU) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  return v;
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
  const int cg = lane % LPR, rr = lane / LPR;
  const int n = n0 + cg * VEC;
  const int valid = max(0, min(VEC, p.N - n));
#pragma unroll 1
  for (int pass = 0; pass < 32 / RPP; ++pass) {
    const int rl = pass * RPP + rr;
    const int row = row0 + rl;
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
    if (p.bias) {
#pragma unroll
      for (int k = 0; k < VEC; ++k)
        if (k < valid) v[k] += p.bias_f32 ? ld_elem<float>(p.bias, n + k) : ld_elem<__nv_bfloat16>(p.bias, n + k);
    }
    if (p.R) {
      float o[VEC];
      ld_vec<T, VEC>(p.R, rb + (int64_t)row * p.ldr + n, valid, p.r_vec, o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] += o[k];
    }
    if (p.act != ACT_NONE) {
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = act_apply(p.act, v[k]);
    }
    if (p.Mk) {
      float o[VEC];
      ld_vec<T, VEC>(p.Mk, mb + (int64_t)row * p.ldm + n, valid, p.m_vec, o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = o[k] > 0.f ? v[k] : 0.f;
    }
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

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, TcParams p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  float* epi = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n * p.batch;
  const int num_kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    fence_barrier_init();
    fence_proxy_async_smem();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        int tm, tn, b;
        tile_coords(t, p, tm, tn, b);
        const int bo = b / p.batch2, bi = b - bo * p.batch2;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err)) goto producer_done;
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if (!p.a_mn) {
            tma_load_4d(sA, &tmA, &full[stage], kb * BK, tm * BM, bi, bo);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_4d(sA + j * 8192, &tmA, &full[stage], tm * BM + j * 64, kb * BK, bi, bo);
          }
          if (!p.b_mn) {
            tma_load_4d(sB, &tmB, &full[stage], kb * BK, tn * BN, bi, bo);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_4d(sB + j * 8192, &tmB, &full[stage], tn * BN + j * 64, kb * BK, bi, bo);
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
    if (lane == 0) {
      const uint32_t idesc = make_idesc(1, 1, 1, p.a_mn != 0, p.b_mn != 0, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aBase = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t bBase = aBase + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = p.a_mn ? make_sw128_desc(aBase + k * 2048, 8192, 1024)
                                       : make_sw128_desc(aBase + k * 32, 16, 1024);
            const uint64_t bd = p.b_mn ? make_sw128_desc(bBase + k * 2048, 8192, 1024)
                                       : make_sw128_desc(bBase + k * 32, 16, 1024);
            mma_f16(d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
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
    // Epilogue warps 2..5.  TMEM lane quarter accessible to a warp = warp % 4.
    // Each 32x32 accumulator chunk is staged through shared memory so that
    // every global access (C, beta*C, bias, residual, ReLU mask) is a
    // coalesced 16-byte access along rows instead of one row per lane.
    const int q = warp & 3;
    float* stg = epi + (warp - 2) * (32 * 33);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn, b;
      tile_coords(t, p, tm, tn, b);
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) break;
      tc_fence_after();
      const int bo = b / p.batch2, bi = b - bo * p.batch2;
      const int64_t cb = (int64_t)bo * p.bsc + (int64_t)bi * p.bsc2;
      const int64_t rb = (int64_t)bo * p.bsr + (int64_t)bi * p.bsr2;
      const int64_t mb = (int64_t)bo * p.bsm + (int64_t)bi * p.bsm2;
      const int row0 = tm * BM + q * 32;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = __uint_as_float(r[j]) * p.alpha;
        __syncwarp();
        const int n0 = tn * BN + c * 32;
        if (n0 < p.N && row0 < p.M) {
          if (p.out_f32) epi_store<float, 4>(p, stg, row0, n0, lane, cb, rb, mb);
          else epi_store<__nv_bfloat16, 8>(p, stg, row0, n0, lane, cb, rb, mb);
        }
        __syncwarp();
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// 4-D bf16 tensor map: dims {d0 (contiguous), d1, inner batch, outer batch},
// strides in elements, box {64, box1, 1, 1}, 128-byte swizzle, zero fill out
// of bounds.
CUtensorMap make_tmap_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1,
                           uint64_t s2, uint64_t s3, uint32_t box1) {
  CUtensorMap m;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1 * 2, s2 * 2, s3 * 2};
  cuuint32_t box[4] = {64, box1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("dlvk: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&dev));
  if (n[dev] == 0) DLVK_CUDA_CHECK(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return n[dev];
}

template <int BN>
void launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& p, int max_ctas, cudaStream_t s) {
  using C = Cfg<BN>;
  static bool attr_set[64] = {false};
  int dev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    DLVK_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    attr_set[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n * p.batch;
  int grid = std::min(tiles, max_ctas > 0 ? max_ctas : sm_count());
  gemm_tc_kernel<BN><<<grid, 192, C::SMEM, s>>>(ta, tb, p);
  DLVK_POST_LAUNCH();
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

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

void gemm_tc(DType out_dt, const GemmArgs& a, cudaStream_t s, uint32_t* err, int max_ctas) {
  DLVK_CHECK(gemm_tc_supported(a), "gemm_tc: unsupported layout/alignment");
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
  const int BN = (a.N >= 256) ? 256 : 128;
  // Unused batch levels get a harmless stride (a multiple of 16 bytes).
  auto pick = [](int64_t cnt, int64_t stride, uint64_t dflt) { return cnt > 1 ? (uint64_t)stride : dflt; };
  CUtensorMap ta, tb;
  if (a_k) {
    const uint64_t d = (uint64_t)a.sam * (uint64_t)a.M;
    ta = make_tmap_bf16(a.A, a.K, a.M, a.batch2, a.batch, a.sam, pick(a.batch2, a.batch2_stride_a, d),
                        pick(a.batch, a.batch_stride_a, d), BM);
  } else {
    const uint64_t d = (uint64_t)a.sak * (uint64_t)a.K;
    ta = make_tmap_bf16(a.A, a.M, a.K, a.batch2, a.batch, a.sak, pick(a.batch2, a.batch2_stride_a, d),
                        pick(a.batch, a.batch_stride_a, d), 64);
  }
  if (b_k) {
    const uint64_t d = (uint64_t)a.sbn * (uint64_t)a.N;
    tb = make_tmap_bf16(a.B, a.K, a.N, a.batch2, a.batch, a.sbn, pick(a.batch2, a.batch2_stride_b, d),
                        pick(a.batch, a.batch_stride_b, d), BN);
  } else {
    const uint64_t d = (uint64_t)a.sbk * (uint64_t)a.K;
    tb = make_tmap_bf16(a.B, a.N, a.K, a.batch2, a.batch, a.sbk, pick(a.batch2, a.batch2_stride_b, d),
                        pick(a.batch, a.batch_stride_b, d), 64);
  }
  TcParams p{};
  p.M = (int)a.M;
  p.N = (int)a.N;
  p.K = (int)a.K;
  p.batch = (int)(a.batch * a.batch2);
  p.batch2 = (int)a.batch2;
  p.tiles_m = (int)((a.M + BM - 1) / BM);
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
  p.act = a.act;
  p.err = err;
  if (BN == 256) launch_tc<256>(ta, tb, p, max_ctas, s);
  else launch_tc<128>(ta, tb, p, max_ctas, s);
}

}  // namespace dlvk
