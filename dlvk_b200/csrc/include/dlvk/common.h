// Common definitions shared by every dlvk_b200 kernel translation unit.
//
// Kernels in this project are plain CUDA (no PyTorch headers).  Each launcher
// takes raw device pointers, sizes and the cudaStream_t to launch on, and
// returns a cudaError_t (or throws std::runtime_error from host checks).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <atomic>
#include <utility>

namespace dlvk {

// Element types understood by the kernels.  Values are stable: they are also
// written into `.dlvk` v2 tensor records.
enum class DType : uint32_t { F32 = 0, BF16 = 1, F16 = 2, I32 = 3, I8 = 4, U8 = 5, I64 = 6 };

// Device-side status codes written to a status word by kernels that can give
// up (bounded waits) or detect bad input (bounds-check build).
enum Status : uint32_t {
  DLVK_OK = 0,
  DLVK_ERR_PEER_TIMEOUT = 1,   // a cross-GPU flag wait ran out of its budget
  DLVK_ERR_BOUNDS = 2,         // DLVK_DEBUG_BOUNDS: an index was out of range
  DLVK_ERR_MBAR_TIMEOUT = 3,   // an mbarrier wait inside a kernel ran out of budget
  DLVK_ERR_BAD_ARG = 4,
};

// Number of kernel launches issued through dlvk launchers (process-wide).
// Used by the bench to report how many of this project's kernels ran.
uint64_t launch_count();
void note_launch(uint64_t n = 1);

[[noreturn]] void throw_cuda(cudaError_t e, const char* what, const char* file, int line);

}  // namespace dlvk

#define DLVK_CUDA_CHECK(expr)                                                    \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) ::dlvk::throw_cuda(_e, #expr, __FILE__, __LINE__);    \
  } while (0)

#define DLVK_CHECK(cond, msg)                                                    \
  do {                                                                           \
    if (!(cond)) throw std::runtime_error(std::string("dlvk: ") + (msg));        \
  } while (0)

namespace dlvk {
// Per-device host caches (kernel attributes, SM counts, error words) are
// fixed arrays of kMaxDevices slots.  current_device_slot() returns the
// current device's ordinal after checking that it fits, so no launcher
// indexes one of those arrays out of bounds.
constexpr int kMaxDevices = 64;
inline int current_device_slot() {
  int dev = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&dev));
  DLVK_CHECK(dev >= 0 && dev < kMaxDevices,
             "device ordinal " + std::to_string(dev) + " is beyond the per-device cache size 64");
  return dev;
}
}  // namespace dlvk

// Launch bookkeeping: every launcher calls this right after its <<<>>>.
#define DLVK_POST_LAUNCH()                                                       \
  do {                                                                           \
    ::dlvk::note_launch();                                                       \
    DLVK_CUDA_CHECK(cudaGetLastError());                                         \
  } while (0)

namespace dlvk {
// Programmatic dependent launch (sm_90+).  A kernel launched through
// launch_pdl() may begin (prologue: barrier init, TMEM allocation, tensor-map
// prefetch) while the previous kernel in the stream is still finishing; it
// must execute pdl_wait() before its first access to global memory, which
// returns once the previous grid has completed and its writes are visible.
// The persistent tensor-core kernels call pdl_trigger() when a CTA has
// finished its work, so their successor's prologue overlaps the tail.
// Opt-in with DLVK_PDL=1; otherwise the launches are ordinary
// stream-serialised ones and the waits return at once.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DLVK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}
}  // namespace dlvk

#ifdef __CUDACC__
namespace dlvk {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `smem` must hold at least 32 floats.  Result is valid in
// every thread.  Fixed reduction order => deterministic.
__device__ __forceinline__ float block_sum(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = (threadIdx.x < nw) ? smem[threadIdx.x] : 0.f;
  if (wid == 0) r = warp_sum(r);
  if (threadIdx.x == 0) smem[0] = r;
  __syncthreads();
  return smem[0];
}
__device__ __forceinline__ float block_max(float v, float* smem) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float r = (threadIdx.x < nw) ? smem[threadIdx.x] : -INFINITY;
  if (wid == 0) r = warp_max(r);
  if (threadIdx.x == 0) smem[0] = r;
  __syncthreads();
  return smem[0];
}

// Philox4x32-10 counter-based generator (Salmon, Moraes, Dror, Shaw:
// "Parallel random numbers: as easy as 1, 2, 3", SC'11).  Multipliers and
// Weyl increments are the ones published in that paper.
struct Philox4 {
  uint4 ctr;
  uint2 key;
};
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += W0;
    k.y += W1;
  }
  return c;
}
// Uniform float in [0,1) from 32 random bits (24-bit mantissa resolution).
__device__ __forceinline__ float u01(uint32_t r) { return (r >> 8) * (1.0f / 16777216.0f); }

}  // namespace dlvk
#endif  // __CUDACC__
