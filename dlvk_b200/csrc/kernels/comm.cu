// Data-parallel gradient all-reduce fused with the optimizer update, over
// NVLink peer memory (P2P loads/stores through IPC-mapped buffers), plus the
// plain P2P all-reduce used by the communication backend.
//
// Replaces the reference's RingAllReduce (src/deployment/ring_all_reduce.cpp:
// 141-271: host-orchestrated "ring" whose transfer step records only a
// pipeline barrier and whose add step is empty) and shaders/
// ring_all_reduce_add.comp (never loaded by any host code).
//
// Protocol for one bucket [start, end) of the flat gradient buffer, epoch e
// (a device counter bumped once per training step):
//   1. ready:  every rank announces "my gradients of this bucket are final"
//              by st.release.sys of e into flags[bucket][0][rank] on every
//              peer, then all CTAs wait (ld.acquire.sys, bounded) until all
//              ranks' ready flags equal e.
//   2. reduce: two-shot -- rank r owns shard r: it sums the shard over all
//              ranks in rank order (fp32, deterministic), scales by 1/world,
//              applies the optimizer to its master/m/v and stores the new
//              compute-dtype parameters into every rank's parameter buffer.
//              one-shot (small buckets) -- every rank reduces the whole
//              bucket itself and updates its own copy; no stores to peers.
//   3. done:   the last CTA of the grid announces "finished reading your
//              gradients / writing your parameters" to every peer and waits
//              for all peers' done flags, so no rank starts its next step
//              while a peer still reads its gradients or writes its params.
// Every wait is bounded by a wall-clock budget; on expiry the kernel records
// DLVK_ERR_PEER_TIMEOUT in the error word and returns.  Peer memory is only
// read with plain per-thread loads (no TMA).
#include "dlvk/common.h"
#include "dlvk/kernels.h"
#include "dlvk/optim_math.h"
#include "dlvk/comm.h"

namespace dlvk {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait until *flag == epoch.  Returns false (and records the timeout) after
// budget_ns.
__device__ bool wait_flag(const uint32_t* flag, uint32_t epoch, uint64_t budget_ns, uint32_t* err) {
  if (ld_acquire_sys(flag) == epoch) return true;
  const uint64_t t0 = gtimer();
  while (true) {
    if (ld_acquire_sys(flag) == epoch) return true;
    if (gtimer() - t0 > budget_ns) {
      atomicCAS(err, 0u, (uint32_t)DLVK_ERR_PEER_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ uint32_t* flag_slot(uint32_t* base, int bucket, int phase, int src, int world) {
  return base + ((int64_t)bucket * 2 + phase) * world + src;
}

template <typename T> struct Pack;  // 16-byte packs
template <> struct Pack<float> { static constexpr int N = 4; };
template <> struct Pack<__nv_bfloat16> { static constexpr int N = 8; };

template <typename T>
__device__ __forceinline__ void load_pack(const T* p, float* out) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int k = 0; k < Pack<T>::N; ++k) out[k] = to_f32(e[k]);
}

// Phase 1 announce + wait.  All CTAs wait; CTA 0 announces.
__device__ bool ready_barrier(const FusedARArgs& a, uint32_t epoch) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(flag_slot(a.peer_flags[threadIdx.x], a.bucket, 0, a.rank, a.world), epoch);
  }
  if (threadIdx.x < a.world) {
    if (!wait_flag(flag_slot(a.my_flags, a.bucket, 0, threadIdx.x, a.world), epoch, a.budget_ns, a.err)) ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// Phase 3: the last CTA to finish announces done and waits for all peers.
__device__ void done_barrier(const FusedARArgs& a, uint32_t epoch) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(a.cta_counter, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!last) return;
  if (threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(flag_slot(a.peer_flags[threadIdx.x], a.bucket, 1, a.rank, a.world), epoch);
    wait_flag(flag_slot(a.my_flags, a.bucket, 1, threadIdx.x, a.world), epoch, a.budget_ns, a.err);
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.cta_counter = 0u;
}

template <typename T> __device__ __forceinline__ float4 load4(const T* base, int64_t vi);
template <> __device__ __forceinline__ float4 load4<float>(const float* base, int64_t vi) {
  return reinterpret_cast<const float4*>(base)[vi];
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* base, int64_t vi) {
  const uint2 u = reinterpret_cast<const uint2*>(base)[vi];
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  return make_float4(a.x, a.y, b.x, b.y);
}
template <typename T> __device__ __forceinline__ void store4(T* base, int64_t vi, const float4& v);
template <> __device__ __forceinline__ void store4<float>(float* base, int64_t vi, const float4& v) {
  reinterpret_cast<float4*>(base)[vi] = v;
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* base, int64_t vi, const float4& v) {
  uint2 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
  h[0] = __floats2bfloat162_rn(v.x, v.y);
  h[1] = __floats2bfloat162_rn(v.z, v.w);
  reinterpret_cast<uint2*>(base)[vi] = u;
}

// Bucket and shard boundaries are multiples of 64 elements (parameter
// offsets in the flat buffers are 256-byte aligned), so the loops below work
// on whole 4-element vectors.  With the world size W a template parameter,
// every peer's U gradient vectors and the local optimizer state of an
// iteration are all issued before the first is consumed, keeping enough bytes
// in flight to cover NVLink latency.  W = 0 is the runtime-world fallback.
template <typename TG, typename TV, int W, int U>
__global__ void __launch_bounds__(128, 6) fused_ar_opt_kernel(FusedARArgs a) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  if (!ready_barrier(a, epoch)) return;
  const OptimHyper h = *a.hyper;
  const float gs = a.scale * h.grad_scale;
  const int world = W > 0 ? W : a.world;
  const int64_t n = a.end - a.start;
  int64_t lo = 0, hi = n;
  if (!a.one_shot) {
    const int64_t shard = ((n + world - 1) / world + 63) / 64 * 64;
    lo = min(n, shard * a.rank);
    hi = min(n, lo + shard);
  }
  const int64_t base = a.start + lo;  // element offset of this rank's range
  const int64_t nvec = (hi - lo) / 4;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float* mst = a.master + base;
  float* mm = a.m ? a.m + base : nullptr;
  float* vv = a.v ? a.v + base : nullptr;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t v0 = tid; v0 < nvec; v0 += stride * U) {
    float4 g[U], w[U], m4[U], v4[U];
    if (W > 0) {
      float4 t[W > 0 ? W : 1][U];
#pragma unroll
      for (int r = 0; r < (W > 0 ? W : 1); ++r) {
        const TG* src = reinterpret_cast<const TG*>(a.peer_grads[r]) + base;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t vi = v0 + u * stride;
          t[r][u] = vi < nvec ? load4<TG>(src, vi) : z4;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = v0 + u * stride;
        w[u] = vi < nvec ? reinterpret_cast<const float4*>(mst)[vi] : z4;
        m4[u] = (mm && vi < nvec) ? reinterpret_cast<const float4*>(mm)[vi] : z4;
        v4[u] = (vv && vi < nvec) ? reinterpret_cast<const float4*>(vv)[vi] : z4;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        g[u] = z4;
#pragma unroll
        for (int r = 0; r < (W > 0 ? W : 1); ++r) {  // rank order: deterministic
          g[u].x += t[r][u].x;
          g[u].y += t[r][u].y;
          g[u].z += t[r][u].z;
          g[u].w += t[r][u].w;
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) g[u] = z4;
      for (int r = 0; r < world; ++r) {
        const TG* src = reinterpret_cast<const TG*>(a.peer_grads[r]) + base;
        float4 t[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t vi = v0 + u * stride;
          t[u] = vi < nvec ? load4<TG>(src, vi) : z4;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          g[u].x += t[u].x;
          g[u].y += t[u].y;
          g[u].z += t[u].z;
          g[u].w += t[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = v0 + u * stride;
        w[u] = vi < nvec ? reinterpret_cast<const float4*>(mst)[vi] : z4;
        m4[u] = (mm && vi < nvec) ? reinterpret_cast<const float4*>(mm)[vi] : z4;
        v4[u] = (vv && vi < nvec) ? reinterpret_cast<const float4*>(vv)[vi] : z4;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t vi = v0 + u * stride;
      if (vi >= nvec) continue;
      opt_apply(a.kind, h, w[u].x, g[u].x * gs, m4[u].x, v4[u].x);
      opt_apply(a.kind, h, w[u].y, g[u].y * gs, m4[u].y, v4[u].y);
      opt_apply(a.kind, h, w[u].z, g[u].z * gs, m4[u].z, v4[u].z);
      opt_apply(a.kind, h, w[u].w, g[u].w * gs, m4[u].w, v4[u].w);
      reinterpret_cast<float4*>(mst)[vi] = w[u];
      if (mm) reinterpret_cast<float4*>(mm)[vi] = m4[u];
      if (vv) reinterpret_cast<float4*>(vv)[vi] = v4[u];
      if (a.values_are_master) {
        // fp32 mode: the master is the compute copy; peers still need it.
        if (!a.one_shot)
          for (int r = 0; r < world; ++r)
            if (r != a.rank) store4<float>(reinterpret_cast<float*>(a.peer_values[r]) + base, vi, w[u]);
      } else {
        const int r0 = a.one_shot ? a.rank : 0, r1 = a.one_shot ? a.rank + 1 : world;
        for (int r = r0; r < r1; ++r) store4<TV>(reinterpret_cast<TV*>(a.peer_values[r]) + base, vi, w[u]);
      }
    }
  }
  done_barrier(a, epoch);
}

template <typename TG, typename TV>
void launch_fused(const FusedARArgs& a, int grid, cudaStream_t s) {
  switch (a.world) {
    case 1: fused_ar_opt_kernel<TG, TV, 1, 2><<<grid, 128, 0, s>>>(a); break;
    case 2: fused_ar_opt_kernel<TG, TV, 2, 2><<<grid, 128, 0, s>>>(a); break;
    case 4: fused_ar_opt_kernel<TG, TV, 4, 1><<<grid, 128, 0, s>>>(a); break;
    case 8: fused_ar_opt_kernel<TG, TV, 8, 1><<<grid, 128, 0, s>>>(a); break;
    default: fused_ar_opt_kernel<TG, TV, 0, 2><<<grid, 128, 0, s>>>(a); break;
  }
}

// Plain two-shot sum all-reduce of [start, end) of a symmetric buffer, in
// place: reduce my shard over all ranks (rank order), store the sum into every
// rank's buffer.  Same flag protocol as the fused kernel.
template <typename T>
__global__ void __launch_bounds__(128, 8) p2p_allreduce_kernel(FusedARArgs a, int average) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  if (!ready_barrier(a, epoch)) return;
  constexpr int V = Pack<T>::N;
  const int64_t n = a.end - a.start;
  const int64_t shard = ((n + a.world - 1) / a.world + 63) / 64 * 64;
  const int64_t lo = min(n, shard * a.rank), hi = min(n, lo + shard);
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float sc = average ? 1.f / a.world : 1.f;
  for (int64_t i = lo + tid * V; i < hi; i += stride * V) {
    const int64_t gi = a.start + i;
    const int cnt = (int)min((int64_t)V, hi - i);
    float acc[V];
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    for (int r = 0; r < a.world; ++r) {
      const T* src = reinterpret_cast<const T*>(a.peer_grads[r]) + gi;
      if (cnt == V) {
        float t[V];
        load_pack<T>(src, t);
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k] += t[k];
      } else {
#pragma unroll
        for (int k = 0; k < V; ++k)
          if (k < cnt) acc[k] += to_f32(src[k]);
      }
    }
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int k = 0; k < V; ++k) e[k] = from_f32<T>(acc[k] * sc);
    // Write back only after every rank has read this shard: the sum goes to a
    // separate region first would need a second buffer; instead each rank
    // writes its own shard's sum to all ranks, which no rank reads again.
    for (int r = 0; r < a.world; ++r) {
      T* dst = reinterpret_cast<T*>(const_cast<void*>(a.peer_grads[r])) + gi;
      if (cnt == V) *reinterpret_cast<uint4*>(dst) = u;
      else
#pragma unroll
        for (int k = 0; k < V; ++k)
          if (k < cnt) dst[k] = e[k];
    }
  }
  done_barrier(a, epoch);
}

}  // namespace

void fused_allreduce_optimizer(const FusedARArgs& a, DType grad_dt, DType value_dt, int ctas, cudaStream_t s) {
  const int64_t n = a.end - a.start;
  if (n <= 0) return;
  DLVK_CHECK(a.world <= 512, "fused all-reduce: world size too large");
  DLVK_CHECK(a.start % 64 == 0 && n % 64 == 0, "fused all-reduce: bucket must be 64-element aligned");
  const int64_t work = a.one_shot ? n : (n + a.world - 1) / a.world;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, (work / 16 + 127) / 128));
  if (grad_dt == DType::F32 && value_dt == DType::BF16) launch_fused<float, __nv_bfloat16>(a, grid, s);
  else if (grad_dt == DType::F32 && value_dt == DType::F32) launch_fused<float, float>(a, grid, s);
  else if (grad_dt == DType::BF16 && value_dt == DType::BF16) launch_fused<__nv_bfloat16, __nv_bfloat16>(a, grid, s);
  else throw std::runtime_error("fused all-reduce: unsupported grad/value dtypes");
  DLVK_POST_LAUNCH();
}

void p2p_allreduce(const FusedARArgs& a, DType dt, bool average, int ctas, cudaStream_t s) {
  const int64_t n = a.end - a.start;
  if (n <= 0) return;
  const int64_t work = (n + a.world - 1) / a.world;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, (work / 8 + 127) / 128));
  if (dt == DType::F32) p2p_allreduce_kernel<float><<<grid, 128, 0, s>>>(a, average ? 1 : 0);
  else if (dt == DType::BF16) p2p_allreduce_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(a, average ? 1 : 0);
  else throw std::runtime_error("p2p all-reduce: unsupported dtype");
  DLVK_POST_LAUNCH();
}

namespace {
// One block waiting on `flag` for `epoch` through the same bounded wait the
// all-reduce kernels use; result[0] = 1 on success, 0 on timeout.
__global__ void wait_flag_probe_kernel(const uint32_t* flag, uint32_t epoch, uint64_t budget_ns, uint32_t* err,
                                       int* result) {
  const bool ok = wait_flag(flag, epoch, budget_ns, err);
  if (threadIdx.x == 0) result[0] = ok ? 1 : 0;
}
}  // namespace

void wait_flag_probe(const uint32_t* flag, uint32_t epoch, uint64_t budget_ns, uint32_t* err, int* result,
                     cudaStream_t s) {
  wait_flag_probe_kernel<<<1, 32, 0, s>>>(flag, epoch, budget_ns, err, result);
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
