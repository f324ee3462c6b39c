// Allocation-free column sums (see dlvk/noalloc.h for who needs this and the
// limits).  No counterpart in the reference framework.
//
// Same two-stage, fixed-order (deterministic) algorithm as dlvk::colsum: row
// chunks of at least 256 rows produce per-chunk partial sums, a second kernel
// adds the chunks in order.  The partials live in a static device array.
#include <mutex>

#include "dlvk/common.h"
#include "dlvk/noalloc.h"

namespace {

static __device__ __align__(256) float g_dlvk_noalloc_scratch[DLVK_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxChunks = 64;
constexpr int kMaxDevices = 64;

std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Per device, with that device current: the device address of the array.
// Host code must not use the symbol itself as a device pointer.
float* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = DLVK_NOALLOC_CUDA_ERROR;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dlvk_noalloc_scratch) != cudaSuccess || p == nullptr) {
      *err = DLVK_NOALLOC_CUDA_ERROR;
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

template <typename T>
__global__ void noalloc_colsum_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t rows_per_chunk,
                                      float scale, float* __restrict__ out, int accumulate,
                                      float* __restrict__ part) {
  __shared__ float sm[8][33];
  const int64_t c = blockIdx.x * 32 + threadIdx.x;
  const int64_t r0 = blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(rows, r0 + rows_per_chunk);
  float acc = 0.f;
  if (c < cols)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += 8) acc += dlvk::to_f32(x[r * cols + c]);
  sm[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y != 0 || c >= cols) return;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += sm[i][threadIdx.x];
  if (gridDim.y > 1) {
    part[blockIdx.y * cols + c] = s;
    return;
  }
  s *= scale;
  out[c] = accumulate ? out[c] + s : s;
}

__global__ void noalloc_colsum_final_kernel(const float* __restrict__ part, int chunks, int64_t cols, float scale,
                                            float* __restrict__ out, int accumulate) {
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += part[k * cols + c];
  s *= scale;
  out[c] = accumulate ? out[c] + s : s;
}

}  // namespace

extern "C" int dlvk_colsum_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, float scale, float* out,
                                   int accumulate, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || rows < 0 || cols < 0 || (dtype != 0 && dtype != 1))
    return DLVK_NOALLOC_BAD_ARG;
  if (cols > DLVK_NOALLOC_MAX_COLS) return DLVK_NOALLOC_TOO_LARGE;
  if (rows == 0 || cols == 0) return DLVK_NOALLOC_OK;
  // An error that earlier, unrelated work left pending on this thread is
  // reported before anything is queued (and left pending for the caller's
  // own handling).  The launch checks below then see only this call's own
  // launches, and the first kernel writes `out` only when it is the sole
  // launch: a DLVK_NOALLOC_CUDA_ERROR return never follows a queued kernel
  // that wrote `out`, so retrying with accumulate = 1 cannot add twice.
  if (cudaPeekAtLastError() != cudaSuccess) return DLVK_NOALLOC_CUDA_ERROR;
  int err = DLVK_NOALLOC_OK;
  float* part = scratch_for_current_device(&err);
  if (part == nullptr) return err;
  int64_t chunks = std::min<int64_t>(kMaxChunks, std::max<int64_t>(1, rows / 256));
  const int64_t rpc = (rows + chunks - 1) / chunks;
  chunks = (rows + rpc - 1) / rpc;
  dim3 block(32, 8), grid((unsigned)((cols + 31) / 32), (unsigned)chunks);
  if (dtype == 0)
    noalloc_colsum_kernel<float><<<grid, block, 0, stream>>>(static_cast<const float*>(x), rows, cols, rpc, scale,
                                                             out, accumulate, part);
  else
    noalloc_colsum_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), rows,
                                                                     cols, rpc, scale, out, accumulate, part);
  if (cudaGetLastError() != cudaSuccess) return DLVK_NOALLOC_CUDA_ERROR;
  dlvk::note_launch();
  if (chunks > 1) {
    noalloc_colsum_final_kernel<<<(unsigned)((cols + 255) / 256), 256, 0, stream>>>(part, (int)chunks, cols, scale,
                                                                                    out, accumulate);
    if (cudaGetLastError() != cudaSuccess) return DLVK_NOALLOC_CUDA_ERROR;
    dlvk::note_launch();
  }
  return DLVK_NOALLOC_OK;
}

extern "C" const char* dlvk_noalloc_error_string(int code) {
  switch (code) {
    case DLVK_NOALLOC_OK: return "ok";
    case DLVK_NOALLOC_BAD_ARG: return "bad argument (null pointer, negative size or unknown dtype)";
    case DLVK_NOALLOC_TOO_LARGE: return "too many columns for the static scratch array (limit DLVK_NOALLOC_MAX_COLS = 16384)";
    case DLVK_NOALLOC_CUDA_ERROR: return "CUDA error (symbol lookup or kernel launch)";
    default: return "unknown error code";
  }
}
