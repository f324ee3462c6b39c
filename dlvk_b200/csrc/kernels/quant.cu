// int8 quantisation kernels and the CUDA-core int8 GEMM used for shapes the
// tensor-core kernel cannot take.
//
// The reference's ModelOptimizer::quantize_model is empty
// (src/optimization/model_optimizer.cpp:30-42) while its QuantizationConfig
// defaults to symmetric, per-channel int8 (include/dlvk/optimization/
// model_optimizer.h:40-47).  Here: weights symmetric per output channel,
// activations symmetric per row (dynamic), int32 accumulation, fp32
// dequantisation fused with bias and activation.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

// One warp per row: scale = max|x| / 127 (1 for an all-zero row),
// q = round-to-nearest(x / scale) clamped to [-127, 127].
template <typename T>
__global__ void quantize_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                     int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scale) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const T* xr = x + r * ldx;
  float mx = 0.f;
  for (int64_t c = lane; c < cols; c += 32) mx = fmaxf(mx, fabsf(to_f32(xr[c])));
  mx = warp_max(mx);
  const float s = mx > 0.f ? mx / 127.f : 1.f;
  const float inv = 1.f / s;
  int8_t* qr = q + r * ldq;
  for (int64_t c = lane; c < cols; c += 32) {
    const float v = fminf(127.f, fmaxf(-127.f, rintf(to_f32(xr[c]) * inv)));
    qr[c] = (int8_t)v;
  }
  if (lane == 0) scale[r] = s;
}

// C[m, n] = act(sum_k A[m,k] * Bt[n,k] * sa[m] * sb[n] + bias[n]); one thread
// per output, 4-byte packed dot products.
template <typename TO>
__global__ void gemm_i8_simt_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ Bt,
                                    const float* __restrict__ sa, const float* __restrict__ sb,
                                    const float* __restrict__ bias, int act, TO* __restrict__ C, int64_t ldc,
                                    int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb) {
  const int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t m = blockIdx.y;
  if (n >= N || m >= M) return;
  const int8_t* a = A + m * lda;
  const int8_t* b = Bt + n * ldb;
  int acc = 0;
  int64_t k = 0;
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 3) == 0)
    for (; k + 4 <= K; k += 4)
      acc = __dp4a(*reinterpret_cast<const int*>(a + k), *reinterpret_cast<const int*>(b + k), acc);
  for (; k < K; ++k) acc += (int)a[k] * (int)b[k];
  float v = (float)acc * sa[m] * sb[n] + (bias ? bias[n] : 0.f);
  if (act == ACT_RELU) v = fmaxf(v, 0.f);
  C[m * ldc + n] = from_f32<TO>(v);
}

}  // namespace

void quantize_rows_int8(DType dt, const void* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* q, int64_t ldq,
                        float* scale, cudaStream_t s) {
  if (rows == 0) return;
  const unsigned g = (unsigned)((rows + 7) / 8);
  if (dt == DType::F32)
    quantize_rows_kernel<float><<<g, 256, 0, s>>>((const float*)x, rows, cols, ldx, q, ldq, scale);
  else if (dt == DType::BF16)
    quantize_rows_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, rows, cols, ldx, q, ldq, scale);
  else
    throw std::runtime_error("dlvk::quantize_rows_int8: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void gemm_i8_simt(const int8_t* A, const int8_t* Bt, const float* sa, const float* sb, const float* bias, int act,
                  void* C, DType out_dt, int64_t ldc, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                  cudaStream_t s) {
  if (M == 0 || N == 0) return;
  dim3 grid((unsigned)((N + 127) / 128), (unsigned)M);
  if (out_dt == DType::F32)
    gemm_i8_simt_kernel<float><<<grid, 128, 0, s>>>(A, Bt, sa, sb, bias, act, (float*)C, ldc, M, N, K, lda, ldb);
  else if (out_dt == DType::BF16)
    gemm_i8_simt_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(A, Bt, sa, sb, bias, act, (__nv_bfloat16*)C, ldc, M, N,
                                                            K, lda, ldb);
  else
    throw std::runtime_error("dlvk::gemm_i8_simt: unsupported output dtype");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
