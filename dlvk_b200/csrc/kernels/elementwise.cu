// Elementwise, activation, broadcast and cast kernels (fp32 and bf16 I/O,
// fp32 math).  These replace the reference's per-op GLSL shaders:
//   relu.comp, relu_backward.comp, sigmoid*.comp, tanh*.comp,
//   tensor_{add,subtract,multiply,divide}.comp, broadcast_add.comp,
//   scalar_multiply.comp, clamp.comp, sqrt.comp
// (reference shaders/*.comp; dispatch in src/tensor/tensor_ops.cpp:47-185,
// 300-463, 2175-2289).  One templated grid-stride kernel per arity, with
// 16-byte vector access when the pointers and length allow it.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

template <typename T> struct Vec;  // 16-byte vector of T
template <> struct Vec<float> { using type = float4; static constexpr int N = 4; };
template <> struct Vec<__nv_bfloat16> { using type = uint4; static constexpr int N = 8; };

template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  using V = typename Vec<T>::type;
  V v = *reinterpret_cast<const V*>(p);
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) out[i] = to_f32(e[i]);
}
template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* in) {
  using V = typename Vec<T>::type;
  V v;
  T* e = reinterpret_cast<T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec<T>::N; ++i) e[i] = from_f32<T>(in[i]);
  *reinterpret_cast<V*>(p) = v;
}

__device__ __forceinline__ float apply_unary(int op, float x, float a, float b) {
  switch (op) {
    case UN_RELU: return x > 0.f ? x : 0.f;
    case UN_SIGMOID: return 1.f / (1.f + expf(-x));
    case UN_TANH: return tanhf(x);
    case UN_SCALE: return x * a;
    case UN_CLAMP: return fminf(fmaxf(x, a), b);
    case UN_SQRT: return sqrtf(x);
    case UN_COPY: return x;
    case UN_SQUARE: return x * x;
    case UN_ADD_SCALAR: return x + a;
    case UN_ABS: return fabsf(x);
    case UN_EXP: return expf(x);
    case UN_LOG: return logf(x);
    case UN_GELU: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
    default: return x;
  }
}

// Binary ops.  DIV keeps the reference's guard: |b| < 1e-8 -> sign(a) * 1e8
// (shaders/tensor_divide.comp:29-34).
__device__ __forceinline__ float apply_binary(int op, float x, float y) {
  switch (op) {
    case BIN_ADD: return x + y;
    case BIN_SUB: return x - y;
    case BIN_MUL: return x * y;
    case BIN_DIV: return fabsf(y) < 1e-8f ? (x >= 0.f ? 1e8f : -1e8f) : x / y;
    case BIN_MAX: return fmaxf(x, y);
    case BIN_MIN: return fminf(x, y);
    // Activation backward ops: x = upstream grad, y = saved tensor.
    case BIN_RELU_BWD: return y > 0.f ? x : 0.f;           // y = forward input or output
    case BIN_SIGMOID_BWD: return x * y * (1.f - y);        // y = sigmoid output
    case BIN_TANH_BWD: return x * (1.f - y * y);           // y = tanh output
    case BIN_GELU_BWD: {                                   // y = forward input
      const float cdf = 0.5f * (1.f + erff(y * 0.70710678118654752f));
      const float pdf = 0.3989422804014327f * expf(-0.5f * y * y);
      return x * (cdf + y * pdf);
    }
    default: return x;
  }
}

template <typename TI, typename TO>
__global__ void unary_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t n, int op,
                             float a, float b, bool vec) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    constexpr int V = Vec<TI>::N < Vec<TO>::N ? Vec<TI>::N : Vec<TO>::N;
    const int64_t nv = n / V;
    for (int64_t i = tid; i < nv; i += stride) {
      float v[8];
#pragma unroll
      for (int j = 0; j < V; ++j) v[j] = to_f32(x[i * V + j]);
#pragma unroll
      for (int j = 0; j < V; ++j) y[i * V + j] = from_f32<TO>(apply_unary(op, v[j], a, b));
    }
    for (int64_t i = nv * V + tid; i < n; i += stride) y[i] = from_f32<TO>(apply_unary(op, to_f32(x[i]), a, b));
  } else {
    for (int64_t i = tid; i < n; i += stride) y[i] = from_f32<TO>(apply_unary(op, to_f32(x[i]), a, b));
  }
}

template <typename T>
__global__ void binary_kernel(const T* __restrict__ x, const T* __restrict__ y, T* __restrict__ z,
                              int64_t n, int op, bool vec) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    constexpr int V = Vec<T>::N;
    const int64_t nv = n / V;
    for (int64_t i = tid; i < nv; i += stride) {
      float a[V], b[V];
      load_vec(x + i * V, a);
      load_vec(y + i * V, b);
#pragma unroll
      for (int j = 0; j < V; ++j) a[j] = apply_binary(op, a[j], b[j]);
      store_vec(z + i * V, a);
    }
    for (int64_t i = nv * V + tid; i < n; i += stride)
      z[i] = from_f32<T>(apply_binary(op, to_f32(x[i]), to_f32(y[i])));
  } else {
    for (int64_t i = tid; i < n; i += stride)
      z[i] = from_f32<T>(apply_binary(op, to_f32(x[i]), to_f32(y[i])));
  }
}

// out[r, c] = act(x[r, c] + bias[c])   (broadcast_add.comp + fused activation)
template <typename T, typename TB>
__global__ void bias_act_kernel(const T* __restrict__ x, const TB* __restrict__ bias, T* __restrict__ out,
                                int64_t rows, int64_t cols, int act) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f32(x[i]) + (bias ? to_f32(bias[i % cols]) : 0.f);
    if (act != UN_COPY) v = apply_unary(act, v, 0.f, 0.f);
    out[i] = from_f32<T>(v);
  }
}

inline int grid_for(int64_t n, int threads = 256) {
  int64_t g = (n + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

void unary(DType dt_in, DType dt_out, const void* x, void* y, int64_t n, int op, float a, float b,
           cudaStream_t s) {
  if (n == 0) return;
  const bool vec = aligned16(x) && aligned16(y);
  const int g = grid_for(n / 4 + 1);
  if (dt_in == DType::F32 && dt_out == DType::F32)
    unary_kernel<float, float><<<g, 256, 0, s>>>((const float*)x, (float*)y, n, op, a, b, vec);
  else if (dt_in == DType::BF16 && dt_out == DType::BF16)
    unary_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n, op, a, b, vec);
  else if (dt_in == DType::F32 && dt_out == DType::BF16)
    unary_kernel<float, __nv_bfloat16><<<g, 256, 0, s>>>((const float*)x, (__nv_bfloat16*)y, n, op, a, b, vec);
  else if (dt_in == DType::BF16 && dt_out == DType::F32)
    unary_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (float*)y, n, op, a, b, vec);
  else
    throw std::runtime_error("dlvk::unary: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void binary(DType dt, const void* x, const void* y, void* z, int64_t n, int op, cudaStream_t s) {
  if (n == 0) return;
  const bool vec = aligned16(x) && aligned16(y) && aligned16(z);
  const int g = grid_for(n / 4 + 1);
  if (dt == DType::F32)
    binary_kernel<float><<<g, 256, 0, s>>>((const float*)x, (const float*)y, (float*)z, n, op, vec);
  else if (dt == DType::BF16)
    binary_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)y,
                                                    (__nv_bfloat16*)z, n, op, vec);
  else
    throw std::runtime_error("dlvk::binary: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void bias_act(DType dt, DType dt_bias, const void* x, const void* bias, void* out, int64_t rows,
              int64_t cols, int act, cudaStream_t s) {
  if (rows * cols == 0) return;
  const int g = grid_for(rows * cols);
  if (dt == DType::F32 && dt_bias == DType::F32)
    bias_act_kernel<float, float><<<g, 256, 0, s>>>((const float*)x, (const float*)bias, (float*)out, rows, cols, act);
  else if (dt == DType::BF16 && dt_bias == DType::F32)
    bias_act_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (const float*)bias,
                                                            (__nv_bfloat16*)out, rows, cols, act);
  else if (dt == DType::BF16 && dt_bias == DType::BF16)
    bias_act_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)bias, (__nv_bfloat16*)out, rows, cols, act);
  else
    throw std::runtime_error("dlvk::bias_act: unsupported dtype");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
