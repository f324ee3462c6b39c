// Reductions, transpose and permute kernels.
// Reference shaders: reduce_sum.comp (a per-workgroup partial only; here a
// full deterministic two-stage reduction), reduce_sum_axis0.comp (column
// sums), transpose.comp, tensor_reshape.comp ([B,S,H*D] <-> [B,H,S,D]);
// dispatch in src/tensor/tensor_ops.cpp:465-610, 2862-2952.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

constexpr int kRedThreads = 512;

// Stage 1: each block reduces a contiguous chunk to one partial (fixed order).
template <typename T>
__global__ void reduce_partial_kernel(const T* __restrict__ x, int64_t n, int op, float* __restrict__ part) {
  __shared__ float sm[32];
  const int64_t chunk = (n + gridDim.x - 1) / gridDim.x;
  const int64_t beg = blockIdx.x * chunk;
  const int64_t end = min(n, beg + chunk);
  float acc = (op == RED_MAX) ? -INFINITY : (op == RED_MIN ? INFINITY : 0.f);
  for (int64_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
    const float v = to_f32(x[i]);
    if (op == RED_SUM) acc += v;
    else if (op == RED_SUMSQ) acc += v * v;
    else if (op == RED_MAX) acc = fmaxf(acc, v);
    else if (op == RED_MIN) acc = fminf(acc, v);
    else if (op == RED_ABSMAX) acc = fmaxf(acc, fabsf(v));
  }
  float r;
  if (op == RED_MAX || op == RED_ABSMAX) r = block_max(acc, sm);
  else if (op == RED_MIN) r = -block_max(-acc, sm);
  else r = block_sum(acc, sm);
  if (threadIdx.x == 0) part[blockIdx.x] = r;
}

__global__ void reduce_final_kernel(const float* __restrict__ part, int nparts, int op, float scale,
                                    float* __restrict__ out) {
  __shared__ float sm[32];
  float acc = (op == RED_MAX || op == RED_ABSMAX) ? -INFINITY : (op == RED_MIN ? INFINITY : 0.f);
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    const float v = part[i];
    if (op == RED_MAX || op == RED_ABSMAX) acc = fmaxf(acc, v);
    else if (op == RED_MIN) acc = fminf(acc, v);
    else acc += v;
  }
  float r;
  if (op == RED_MAX || op == RED_ABSMAX) r = block_max(acc, sm);
  else if (op == RED_MIN) r = -block_max(-acc, sm);
  else r = block_sum(acc, sm);
  if (threadIdx.x == 0) out[0] = r * scale;
}

// out[c] = scale * sum_r x[r, c]  (reduce_sum_axis0.comp).  Block = 32 x 8
// threads owning 32 columns; blockIdx.y selects a chunk of rows.  With one
// chunk the block writes the result, otherwise a per-chunk partial that
// colsum_final_kernel sums in chunk order (deterministic).
template <typename T, typename TO>
__global__ void colsum_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, float scale,
                              TO* __restrict__ out, bool accumulate, float* __restrict__ partial,
                              int64_t rows_per_chunk) {
  __shared__ float sm[8][33];
  const int64_t c = blockIdx.x * 32 + threadIdx.x;
  const int64_t r0 = blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(rows, r0 + rows_per_chunk);
  float acc = 0.f;
  if (c < cols)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) acc += to_f32(x[r * cols + c]);
  sm[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && c < cols) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += sm[i][threadIdx.x];
    if (gridDim.y > 1) {
      partial[blockIdx.y * cols + c] = s;
      return;
    }
    s *= scale;
    if (accumulate) s += to_f32(out[c]);
    out[c] = from_f32<TO>(s);
  }
}

template <typename TO>
__global__ void colsum_final_kernel(const float* __restrict__ partial, int chunks, int64_t cols, float scale,
                                    TO* __restrict__ out, bool accumulate) {
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += partial[k * cols + c];
  s *= scale;
  if (accumulate) s += to_f32(out[c]);
  out[c] = from_f32<TO>(s);
}

// out[c] = scale * sum_k partial[k, c] (+ out[c]) for many chunks: 32 columns
// per block, 8 lanes per column each summing every 8th chunk, then a fixed
// tree (deterministic).
__global__ void colsum_partials_kernel(const float* __restrict__ partial, int64_t chunks, int64_t cols, float scale,
                                       float* __restrict__ out, bool accumulate) {
  __shared__ float sm[8][33];
  const int64_t c = blockIdx.x * 32 + threadIdx.x;
  float acc = 0.f;
  if (c < cols)
    for (int64_t k = threadIdx.y; k < chunks; k += 8) acc += partial[k * cols + c];
  sm[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y != 0 || c >= cols) return;
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s2 += sm[i][threadIdx.x];
  s2 *= scale;
  out[c] = accumulate ? out[c] + s2 : s2;
}

// out[r] = scale * sum_c x[r, c]   (row sums, one warp per row)
template <typename T>
__global__ void rowsum_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, float scale,
                              float* __restrict__ out) {
  const int64_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float acc = 0.f;
  const T* xr = x + r * cols;
  constexpr int EPV = 16 / sizeof(T);
  if (cols % EPV == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // 16-byte vectors; each lane keeps two in flight
    const uint4* v = reinterpret_cast<const uint4*>(xr);
    const int64_t nv = cols / EPV;
    int64_t i = lane;
    for (; i + 32 < nv; i += 64) {
      const uint4 a = v[i], b = v[i + 32];
      const T* ea = reinterpret_cast<const T*>(&a);
      const T* eb = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int k = 0; k < EPV; ++k) acc += to_f32(ea[k]) + to_f32(eb[k]);
    }
    for (; i < nv; i += 32) {
      const uint4 a = v[i];
      const T* ea = reinterpret_cast<const T*>(&a);
#pragma unroll
      for (int k = 0; k < EPV; ++k) acc += to_f32(ea[k]);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) acc += to_f32(xr[c]);
  }
  acc = warp_sum(acc);
  if (lane == 0) out[r] = acc * scale;
}

// Batched 2-D transpose through a 32x33 shared tile.
template <typename T>
__global__ void transpose_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int64_t cols) {
  __shared__ T tile[32][33];
  const int64_t b = blockIdx.z;
  x += b * rows * cols;
  y += b * rows * cols;
  const int64_t c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = x[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) y[c * rows + r] = tile[threadIdx.x][i];
  }
}

// General 4-D permute: out[o0,o1,o2,o3] = in[...] with `perm` mapping output
// dims to input dims (tensor_reshape.comp generalised).
template <typename T>
__global__ void permute4_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n, int4 in_dims,
                                int4 perm) {
  const int64_t ist[4] = {(int64_t)in_dims.y * in_dims.z * in_dims.w, (int64_t)in_dims.z * in_dims.w,
                          (int64_t)in_dims.w, 1};
  const int idim[4] = {in_dims.x, in_dims.y, in_dims.z, in_dims.w};
  const int p[4] = {perm.x, perm.y, perm.z, perm.w};
  const int od[4] = {idim[p[0]], idim[p[1]], idim[p[2]], idim[p[3]]};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i;
    int64_t src = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      const int64_t idx = rem % od[d];
      rem /= od[d];
      src += idx * ist[p[d]];
    }
    y[i] = x[src];
  }
}

}  // namespace

int reduce_scratch_floats() { return 1024; }

void reduce(DType dt, const void* x, int64_t n, int op, float scale, float* out, float* scratch,
            cudaStream_t s) {
  int blocks = (int)std::min<int64_t>(1024, (n + kRedThreads * 8 - 1) / (kRedThreads * 8));
  if (blocks < 1) blocks = 1;
  if (dt == DType::F32)
    reduce_partial_kernel<float><<<blocks, kRedThreads, 0, s>>>((const float*)x, n, op, scratch);
  else if (dt == DType::BF16)
    reduce_partial_kernel<__nv_bfloat16><<<blocks, kRedThreads, 0, s>>>((const __nv_bfloat16*)x, n, op, scratch);
  else
    throw std::runtime_error("dlvk::reduce: unsupported dtype");
  DLVK_POST_LAUNCH();
  reduce_final_kernel<<<1, 1024, 0, s>>>(scratch, blocks, op, scale, out);
  DLVK_POST_LAUNCH();
}

int64_t colsum_scratch_floats(int64_t rows, int64_t cols) {
  const int64_t chunks = std::min<int64_t>(64, std::max<int64_t>(1, rows / 256));
  return chunks > 1 ? chunks * cols : 0;
}

void colsum(DType dt, DType dt_out, const void* x, int64_t rows, int64_t cols, float scale, void* out,
            bool accumulate, float* scratch, cudaStream_t s) {
  int64_t chunks = scratch ? std::min<int64_t>(64, std::max<int64_t>(1, rows / 256)) : 1;
  const int64_t rpc = (rows + chunks - 1) / std::max<int64_t>(chunks, 1);
  chunks = std::max<int64_t>(1, (rows + rpc - 1) / std::max<int64_t>(rpc, 1));
  dim3 block(32, 8), grid((unsigned)((cols + 31) / 32), (unsigned)chunks);
#define DLVK_COLSUM(TI, TOUT)                                                                                   \
  do {                                                                                                          \
    colsum_kernel<TI, TOUT><<<grid, block, 0, s>>>((const TI*)x, rows, cols, scale, (TOUT*)out, accumulate, scratch, \
                                                   rpc);                                                          \
    DLVK_POST_LAUNCH();                                                                                          \
    if (chunks > 1) {                                                                                            \
      colsum_final_kernel<TOUT><<<(unsigned)((cols + 255) / 256), 256, 0, s>>>(scratch, (int)chunks, cols, scale,  \
                                                                               (TOUT*)out, accumulate);          \
      DLVK_POST_LAUNCH();                                                                                        \
    }                                                                                                            \
  } while (0)
  if (dt == DType::F32 && dt_out == DType::F32) DLVK_COLSUM(float, float);
  else if (dt == DType::BF16 && dt_out == DType::F32) DLVK_COLSUM(__nv_bfloat16, float);
  else if (dt == DType::BF16 && dt_out == DType::BF16) DLVK_COLSUM(__nv_bfloat16, __nv_bfloat16);
  else throw std::runtime_error("dlvk::colsum: unsupported dtype");
#undef DLVK_COLSUM
}

void colsum_partials(const float* partial, int64_t chunks, int64_t cols, float scale, float* out, bool accumulate,
                     cudaStream_t s) {
  colsum_partials_kernel<<<(unsigned)((cols + 31) / 32), dim3(32, 8), 0, s>>>(partial, chunks, cols, scale, out,
                                                                            accumulate);
  DLVK_POST_LAUNCH();
}

void rowsum(DType dt, const void* x, int64_t rows, int64_t cols, float scale, float* out, cudaStream_t s) {
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  if (dt == DType::F32)
    rowsum_kernel<float><<<grid, wpb * 32, 0, s>>>((const float*)x, rows, cols, scale, out);
  else if (dt == DType::BF16)
    rowsum_kernel<__nv_bfloat16><<<grid, wpb * 32, 0, s>>>((const __nv_bfloat16*)x, rows, cols, scale, out);
  else
    throw std::runtime_error("dlvk::rowsum: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void transpose2d(DType dt, const void* x, void* y, int64_t batch, int64_t rows, int64_t cols, cudaStream_t s) {
  dim3 block(32, 8), grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
  if (dt == DType::F32)
    transpose_kernel<float><<<grid, block, 0, s>>>((const float*)x, (float*)y, rows, cols);
  else if (dt == DType::BF16)
    transpose_kernel<__nv_bfloat16><<<grid, block, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, cols);
  else if (dt == DType::I32)
    transpose_kernel<int><<<grid, block, 0, s>>>((const int*)x, (int*)y, rows, cols);
  else
    throw std::runtime_error("dlvk::transpose2d: unsupported dtype");
  DLVK_POST_LAUNCH();
}

void permute4(DType dt, const void* x, void* y, const int* in_dims, const int* perm, cudaStream_t s) {
  const int64_t n = (int64_t)in_dims[0] * in_dims[1] * in_dims[2] * in_dims[3];
  if (n == 0) return;
  const int4 d = make_int4(in_dims[0], in_dims[1], in_dims[2], in_dims[3]);
  const int4 p = make_int4(perm[0], perm[1], perm[2], perm[3]);
  const unsigned g = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 32);
  if (dt == DType::F32)
    permute4_kernel<float><<<g, 256, 0, s>>>((const float*)x, (float*)y, n, d, p);
  else if (dt == DType::BF16)
    permute4_kernel<__nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n, d, p);
  else
    throw std::runtime_error("dlvk::permute4: unsupported dtype");
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
