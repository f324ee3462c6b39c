// General strided/batched GEMM on the CUDA cores (fp32 FFMA), used for fp32
// mode and for shapes the tensor-core path cannot take (row pitches that are
// not 16-byte multiples, tiny N such as the 128->10 classifier).
//
// Reference: shaders/matrix_multiply.comp:23-37 (one thread per output),
// shaders/batch_matrix_multiply.comp:33-86 (16x16 shared tiles); dispatch in
// src/tensor/tensor_ops.cpp:187-298.  Here: 64x64 block tile, 16-deep K
// slices in shared memory, 4x4 register micro-tile per thread, fused
// alpha/beta, bias and activation epilogue.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

// SPLIT: blockIdx.z is a K slice [z * kper, (z + 1) * kper) of a 2-D GEMM and
// the block writes its raw fp32 partial tile to ws[z] ([M][N]);
// simt_splitk_reduce_kernel applies the epilogue.
template <typename TA, typename TC, bool SPLIT = false>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs a, float* __restrict__ ws = nullptr,
                                                        int64_t kper = 0) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int64_t bz = SPLIT ? 0 : blockIdx.z;
  const int64_t kbeg = SPLIT ? (int64_t)blockIdx.z * kper : 0;
  const int64_t kend = SPLIT ? min(a.K, kbeg + kper) : a.K;
  const int64_t bo = bz / a.batch2, bi = bz - bo * a.batch2;
  const TA* A = reinterpret_cast<const TA*>(a.A) + bo * a.batch_stride_a + bi * a.batch2_stride_a;
  const TA* B = reinterpret_cast<const TA*>(a.B) + bo * a.batch_stride_b + bi * a.batch2_stride_b;
  TC* C = reinterpret_cast<TC*>(a.C) + bo * a.batch_stride_c + bi * a.batch2_stride_c;
  const TC* R = a.residual ? reinterpret_cast<const TC*>(a.residual) + bo * a.batch_stride_r + bi * a.batch2_stride_r
                           : nullptr;
  const TC* Mk = a.relu_mask ? reinterpret_cast<const TC*>(a.relu_mask) + bo * a.batch_stride_m + bi * a.batch2_stride_m
                             : nullptr;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads
  float acc[4][4] = {};
  // The next K slice is loaded into registers while the current one is
  // multiplied out of shared memory, so each block pays the global-load
  // latency once instead of once per slice (small GEMMs run few blocks).
  float ra[4], rb[4];
  auto load = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = threadIdx.x + i * 256;
      // A: choose the mapping that keeps the contiguous dimension on threadIdx.
      int mm, kk;
      if (a.sak == 1) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
      const int64_t gm = m0 + mm, gk = k0 + kk;
      ra[i] = (gm < a.M && gk < kend) ? to_f32(A[gm * a.sam + gk * a.sak]) : 0.f;
      int nn, kb;
      if (a.sbn == 1) { nn = e % BN; kb = e / BN; } else { kb = e % BK; nn = e / BK; }
      const int64_t gn = n0 + nn, gkb = k0 + kb;
      rb[i] = (gn < a.N && gkb < kend) ? to_f32(B[gkb * a.sbk + gn * a.sbn]) : 0.f;
    }
  };
  load(kbeg);
  for (int64_t k0 = kbeg; k0 < kend; k0 += BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = threadIdx.x + i * 256;
      int mm, kk;
      if (a.sak == 1) { kk = e % BK; mm = e / BK; } else { mm = e % BM; kk = e / BM; }
      As[kk][mm] = ra[i];
      int nn, kb;
      if (a.sbn == 1) { nn = e % BN; kb = e / BN; } else { kb = e % BK; nn = e / BK; }
      Bs[kb][nn] = rb[i];
    }
    __syncthreads();
    if (k0 + BK < kend) load(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  if (SPLIT) {
    float* wz = ws + (int64_t)blockIdx.z * a.M * a.N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t gm = m0 + ty * 4 + i;
      if (gm >= a.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn = n0 + tx * 4 + j;
        if (gn < a.N) wz[gm * a.N + gn] = acc[i][j];
      }
    }
    return;
  }
  // Epilogue.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn >= a.N) continue;
      float v = a.alpha * acc[i][j];
      TC* cp = C + gm * a.ldc + gn;
      if (a.beta != 0.f) v += a.beta * to_f32(*cp);
      if (a.bias) {
        v += (a.bias_dtype == (int)DType::F32) ? reinterpret_cast<const float*>(a.bias)[gn]
                                               : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[gn]);
      }
      if (R) v += to_f32(R[gm * a.ldr + gn]);
      if (a.act == ACT_RELU) v = fmaxf(v, 0.f);
      else if (a.act == ACT_GELU) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
      if (Mk && !(to_f32(Mk[gm * a.ldm + gn]) > 0.f)) v = 0.f;
      if (a.relu_bits && !((a.relu_bits[gm * a.ldbits + (gn >> 5)] >> (gn & 31)) & 1u)) v = 0.f;
      // the caller clears the bitmask before this path
      if (a.relu_bits_out && v > 0.f) atomicOr(&a.relu_bits_out[gm * a.ldbits + (gn >> 5)], 1u << (gn & 31));
      *cp = from_f32<TC>(v);
    }
  }
}

// Split-K finish: C = act(alpha * sum_z ws[z] + beta * C + bias), summed in
// slice order (deterministic).
template <typename TC>
__global__ void simt_splitk_reduce_kernel(const float* __restrict__ ws, int splits, GemmArgs a) {
  const int64_t mn = a.M * a.N;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < mn; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t gm = idx / a.N, gn = idx - gm * a.N;
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += ws[(int64_t)z * mn + idx];
    v *= a.alpha;
    TC* cp = reinterpret_cast<TC*>(a.C) + gm * a.ldc + gn;
    if (a.beta != 0.f) v += a.beta * to_f32(*cp);
    if (a.bias) {
      v += (a.bias_dtype == (int)DType::F32) ? reinterpret_cast<const float*>(a.bias)[gn]
                                             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[gn]);
    }
    if (a.act == ACT_RELU) v = fmaxf(v, 0.f);
    else if (a.act == ACT_GELU) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    *cp = from_f32<TC>(v);
  }
}

// Split-K factor for a small 2-D GEMM with a plain epilogue: K slices of at
// least four 16-deep steps until about 148 blocks run; 1 = no split.
int simt_splits(const GemmArgs& a) {
  if (a.batch * a.batch2 != 1 || a.residual || a.relu_mask || a.relu_bits || a.relu_bits_out) return 1;
  const int64_t blocks = ((a.N + BN - 1) / BN) * ((a.M + BM - 1) / BM);
  if (blocks >= 48) return 1;
  const int64_t by_k = a.K / (4 * BK);
  const int64_t by_blocks = (148 + blocks - 1) / blocks;
  return (int)std::max<int64_t>(1, std::min<int64_t>(16, std::min(by_k, by_blocks)));
}

}  // namespace

int64_t gemm_simt_workspace_floats(const GemmArgs& a) {
  const int sp = simt_splits(a);
  return sp > 1 ? (int64_t)sp * a.M * a.N : 0;
}

void gemm_simt(DType in_dt, DType out_dt, const GemmArgs& a, cudaStream_t s, float* ws, int64_t ws_floats) {
  if (a.M == 0 || a.N == 0) return;
  const int sp = ws ? simt_splits(a) : 1;
  if (sp > 1 && ws_floats >= (int64_t)sp * a.M * a.N) {
    int64_t kper = (a.K + sp - 1) / sp;
    kper = (kper + BK - 1) / BK * BK;
    const int splits = (int)((a.K + kper - 1) / kper);
    dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM), (unsigned)splits);
    const int rg = (int)std::min<int64_t>((a.M * a.N + 255) / 256, 148 * 8);
    auto run = [&](auto kern, auto red) {
      kern<<<grid, 256, 0, s>>>(a, ws, kper);
      DLVK_POST_LAUNCH();
      red<<<rg, 256, 0, s>>>(ws, splits, a);
      DLVK_POST_LAUNCH();
    };
    if (in_dt == DType::F32 && out_dt == DType::F32)
      run(gemm_simt_kernel<float, float, true>, simt_splitk_reduce_kernel<float>);
    else if (in_dt == DType::BF16 && out_dt == DType::BF16)
      run(gemm_simt_kernel<__nv_bfloat16, __nv_bfloat16, true>, simt_splitk_reduce_kernel<__nv_bfloat16>);
    else if (in_dt == DType::BF16 && out_dt == DType::F32)
      run(gemm_simt_kernel<__nv_bfloat16, float, true>, simt_splitk_reduce_kernel<float>);
    else if (in_dt == DType::F32 && out_dt == DType::BF16)
      run(gemm_simt_kernel<float, __nv_bfloat16, true>, simt_splitk_reduce_kernel<__nv_bfloat16>);
    else
      throw std::runtime_error("dlvk::gemm_simt: unsupported dtype combination");
    return;
  }
  DLVK_CHECK(a.row_bias == nullptr, "gemm_simt: per-row bias is a tensor-core-path option");
  dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM), (unsigned)(a.batch * a.batch2));
  if (in_dt == DType::F32 && out_dt == DType::F32)
    gemm_simt_kernel<float, float><<<grid, 256, 0, s>>>(a);
  else if (in_dt == DType::BF16 && out_dt == DType::BF16)
    gemm_simt_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, s>>>(a);
  else if (in_dt == DType::BF16 && out_dt == DType::F32)
    gemm_simt_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>(a);
  else if (in_dt == DType::F32 && out_dt == DType::BF16)
    gemm_simt_kernel<float, __nv_bfloat16><<<grid, 256, 0, s>>>(a);
  else
    throw std::runtime_error("dlvk::gemm_simt: unsupported dtype combination");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
