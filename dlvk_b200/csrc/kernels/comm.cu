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

// ---------------------------------------------------------------- NVLS
// multimem operations on NVLink-multicast addresses: the NVSwitch reduces the
// loads over every bound rank's memory and replicates the stores.
__device__ __forceinline__ float4 multimem_ld_reduce_f32x4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void multimem_st_f32x4(float* mc, const float4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
// Orders this thread's accesses through one virtual alias of memory (the
// unicast or the multicast mapping) against its accesses through the other.
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Eight bf16 (16 bytes) stored as four 32-bit lanes: the store moves bits.
__device__ __forceinline__ void multimem_st_bf16x8(__nv_bfloat16* mc, const float4& v0, const float4& v1) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v0.x, v0.y), b = __floats2bfloat162_rn(v0.z, v0.w);
  const __nv_bfloat162 c = __floats2bfloat162_rn(v1.x, v1.y), d = __floats2bfloat162_rn(v1.z, v1.w);
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(__uint_as_float(*reinterpret_cast<const uint32_t*>(&a))),
               "f"(__uint_as_float(*reinterpret_cast<const uint32_t*>(&b))),
               "f"(__uint_as_float(*reinterpret_cast<const uint32_t*>(&c))),
               "f"(__uint_as_float(*reinterpret_cast<const uint32_t*>(&d)))
               : "memory");
}

// NVLS two-shot: my shard's gradients summed by the switch (multimem
// ld_reduce through the multicast mapping), the optimizer applied, and the
// new parameters multicast to every rank with one store.  A thread handles
// units of eight consecutive elements (two 16-byte reduce loads, one 16-byte
// multicast store of bf16 parameters), U units in flight.  The range and the
// shards are multiples of 8 elements (checked on the host).
template <typename TV, int U>
__global__ void __launch_bounds__(128, 4) fused_nvls_ar_opt_kernel(FusedARArgs a) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  if (!ready_barrier(a, epoch)) return;
  fence_proxy_alias();  // the peers' gradients were written through their unicast mappings
  const OptimHyper h = *a.hyper;
  const float gs = a.scale * h.grad_scale;
  const int64_t n = a.end - a.start;
  const int64_t shard = ((n + a.world - 1) / a.world + 63) / 64 * 64;
  const int64_t lo = min(n, shard * a.rank), hi = min(n, lo + shard);
  const int64_t base = a.start + lo;
  const int64_t nunit = (hi - lo) / 8;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float* mg = reinterpret_cast<const float*>(a.mc_grads) + base;
  float4* mst = reinterpret_cast<float4*>(a.master + base);
  float4* mm = a.m ? reinterpret_cast<float4*>(a.m + base) : nullptr;
  float4* vv = a.v ? reinterpret_cast<float4*>(a.v + base) : nullptr;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t u0 = tid; u0 < nunit; u0 += stride * U) {
    float4 g[U][2], w[U][2], m4[U][2], v4[U][2];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t ui = u0 + u * stride;
      const bool on = ui < nunit;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t q = ui * 2 + e;  // float4 index
        g[u][e] = on ? multimem_ld_reduce_f32x4(mg + q * 4) : z4;
        w[u][e] = on ? mst[q] : z4;
        m4[u][e] = (mm && on) ? mm[q] : z4;
        v4[u][e] = (vv && on) ? vv[q] : z4;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t ui = u0 + u * stride;
      if (ui >= nunit) continue;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        opt_apply(a.kind, h, w[u][e].x, g[u][e].x * gs, m4[u][e].x, v4[u][e].x);
        opt_apply(a.kind, h, w[u][e].y, g[u][e].y * gs, m4[u][e].y, v4[u][e].y);
        opt_apply(a.kind, h, w[u][e].z, g[u][e].z * gs, m4[u][e].z, v4[u][e].z);
        opt_apply(a.kind, h, w[u][e].w, g[u][e].w * gs, m4[u][e].w, v4[u][e].w);
        if (mm) mm[ui * 2 + e] = m4[u][e];
        if (vv) vv[ui * 2 + e] = v4[u][e];
      }
      if (a.values_are_master) {
        // fp32 mode: the master is the compute copy and lives in the
        // multicast buffer; one store reaches every rank (this one included).
        float* mv = reinterpret_cast<float*>(a.mc_values) + base + ui * 8;
        multimem_st_f32x4(mv, w[u][0]);
        multimem_st_f32x4(mv + 4, w[u][1]);
      } else {
        mst[ui * 2] = w[u][0];
        mst[ui * 2 + 1] = w[u][1];
        multimem_st_bf16x8(reinterpret_cast<__nv_bfloat16*>(a.mc_values) + base + ui * 8, w[u][0], w[u][1]);
      }
    }
  }
  fence_proxy_alias();  // peers will read the new parameters through their unicast mappings
  done_barrier(a, epoch);
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

// Push two-shot: CTA c of every rank handles chunk c of every rank's shard,
// as PUSH_SUB sub-chunks.
//   A. push:   for each sub-chunk s and each peer k (starting at rank+1, so
//              the ranks' stores spread over all peers), store my gradients
//              of sub-chunk s of chunk c of k's shard into k's receive slot
//              for me, fence, and set k's flag [cbucket][c][s][rank] = epoch.
//   B. reduce: for each sub-chunk, wait (bounded) for the flags of all
//              peers; sum it over the ranks in rank order (my own gradients
//              for my rank, the receive slots for the others), apply the
//              optimizer and store the new parameters into every rank's
//              buffer.  The stores of the last sub-chunks drain over NVLink
//              while the first ones are reduced.
//   C. done:   as in the pull kernels.
// There is no global ready barrier: stream order makes my gradients final
// before the kernel starts, and an owner waits only for the sub-chunks it
// reduces.  All NVLink traffic is stores and every load is local.  The grid
// is sized to be resident at once (one wave), so the waits never depend on
// a CTA that has not been scheduled.
template <typename TG, typename TV, int W, int U>
__global__ void __launch_bounds__(256, 2) fused_push_ar_opt_kernel(FusedARArgs a) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  const int world = W > 0 ? W : a.world;
  const int me = a.rank;
  const int64_t n = a.end - a.start;
  const int64_t shard = ((n + world - 1) / world + 63) / 64 * 64;
  const int64_t c0 = (int64_t)blockIdx.x * a.chunk;
  const int64_t sub = ((a.chunk + PUSH_SUB - 1) / PUSH_SUB + 63) / 64 * 64;
  const int nt = blockDim.x;
  // [lo, lo + len) of rank k's shard covered by sub-chunk s of this CTA.
  auto sub_range = [&](int k, int s, int64_t& lo) -> int64_t {
    const int64_t klen = min(n, shard * (k + 1)) - min(n, shard * k);
    const int64_t cend = min(klen, c0 + a.chunk);
    lo = c0 + s * sub;
    return max((int64_t)0, min(cend, lo + sub) - lo);
  };
  auto flag_at = [&](uint32_t* base, int s, int src) {
    return base + ((int64_t)a.cbucket * PUSH_MAX_CHUNKS + (int64_t)blockIdx.x * PUSH_SUB + s) * world + src;
  };

  // A. push my slices of the peers' shards.
  for (int s = 0; s < PUSH_SUB; ++s) {
    for (int d = 1; d < world; ++d) {
      const int k = (me + d) % world;
      int64_t lo;
      const int64_t len = sub_range(k, s, lo);
      if (len <= 0) continue;
      const int slot = (me - k - 1 + world) % world;
      const uint4* src =
          reinterpret_cast<const uint4*>(reinterpret_cast<const TG*>(a.peer_grads[me]) + a.start + shard * k + lo);
      uint4* dst =
          reinterpret_cast<uint4*>(reinterpret_cast<TG*>(a.peer_recv[k]) + slot * a.recv_slot + a.recv_off + lo);
      const int64_t nv = len * (int64_t)sizeof(TG) / 16;
      constexpr int UA = 4;
      for (int64_t i = threadIdx.x; i < nv; i += (int64_t)nt * UA) {
        uint4 t[UA];
#pragma unroll
        for (int u = 0; u < UA; ++u) {
          const int64_t j = i + (int64_t)u * nt;
          if (j < nv) t[u] = src[j];
        }
#pragma unroll
        for (int u = 0; u < UA; ++u) {
          const int64_t j = i + (int64_t)u * nt;
          if (j < nv) dst[j] = t[u];
        }
      }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < world && (int)threadIdx.x != me) st_release_sys(flag_at(a.peer_cflags[threadIdx.x], s, me), epoch);
  }

  // B. per sub-chunk: wait for the peers' slices, reduce, update, store.
  __shared__ int ok;
  const OptimHyper h = *a.hyper;
  const float gs = a.scale * h.grad_scale;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < PUSH_SUB; ++s) {
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < world && (int)threadIdx.x != me)
      if (!wait_flag(flag_at(a.my_cflags, s, threadIdx.x), epoch, a.budget_ns, a.err)) ok = 0;
    __syncthreads();
    if (!ok) break;
    int64_t lo;
    const int64_t nvec = sub_range(me, s, lo) / 4;
    const int64_t base = a.start + shard * me + lo;  // element offset in the flat buffers
    float* mst = a.master + base;
    float* mm = a.m ? a.m + base : nullptr;
    float* vv = a.v ? a.v + base : nullptr;
    const TG* own = reinterpret_cast<const TG*>(a.peer_grads[me]) + base;
    const TG* recv = reinterpret_cast<const TG*>(a.my_recv) + a.recv_off + lo;
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += (int64_t)nt * U) {
      float4 g[U], w[U], m4[U], v4[U];
#pragma unroll
      for (int u = 0; u < U; ++u) g[u] = z4;
      auto add_rank = [&](int r) {
        const TG* src = r == me ? own : recv + (int64_t)((r - me - 1 + world) % world) * a.recv_slot;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t vi = v0 + (int64_t)u * nt;
          const float4 t = vi < nvec ? load4<TG>(src, vi) : z4;
          g[u].x += t.x;
          g[u].y += t.y;
          g[u].z += t.z;
          g[u].w += t.w;
        }
      };
      if constexpr (W > 0) {
#pragma unroll
        for (int r = 0; r < W; ++r) add_rank(r);  // rank order: deterministic
      } else {
        for (int r = 0; r < world; ++r) add_rank(r);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = v0 + (int64_t)u * nt;
        w[u] = vi < nvec ? reinterpret_cast<const float4*>(mst)[vi] : z4;
        m4[u] = (mm && vi < nvec) ? reinterpret_cast<const float4*>(mm)[vi] : z4;
        v4[u] = (vv && vi < nvec) ? reinterpret_cast<const float4*>(vv)[vi] : z4;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t vi = v0 + (int64_t)u * nt;
        if (vi >= nvec) continue;
        opt_apply(a.kind, h, w[u].x, g[u].x * gs, m4[u].x, v4[u].x);
        opt_apply(a.kind, h, w[u].y, g[u].y * gs, m4[u].y, v4[u].y);
        opt_apply(a.kind, h, w[u].z, g[u].z * gs, m4[u].z, v4[u].z);
        opt_apply(a.kind, h, w[u].w, g[u].w * gs, m4[u].w, v4[u].w);
        reinterpret_cast<float4*>(mst)[vi] = w[u];
        if (mm) reinterpret_cast<float4*>(mm)[vi] = m4[u];
        if (vv) reinterpret_cast<float4*>(vv)[vi] = v4[u];
        for (int d = 0; d < world; ++d) {
          const int r = (me + 1 + d) % world;
          if (a.values_are_master) {
            if (r != me) store4<float>(reinterpret_cast<float*>(a.peer_values[r]) + base, vi, w[u]);
          } else {
            store4<TV>(reinterpret_cast<TV*>(a.peer_values[r]) + base, vi, w[u]);
          }
        }
      }
    }
  }
  done_barrier(a, epoch);
}

// LL one-shot.  Element pair i of the bucket travels as two 8-byte words
// {value bits, epoch}; a 64-bit aligned store is single-copy atomic, so a
// reader that sees the epoch also sees the value.  Words live in
// [parity = epoch & 1][slot][ll_off + i]; a writer can reuse a parity only
// two epochs later, after its own next kernel, which needs this rank's next
// words, which this rank sends only after finishing the current kernel.
__device__ __forceinline__ void st_ll2(void* p, float a, float b, uint32_t e) {
  const uint64_t w0 = (uint64_t)__float_as_uint(a) | ((uint64_t)e << 32);
  const uint64_t w1 = (uint64_t)__float_as_uint(b) | ((uint64_t)e << 32);
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ void ld_ll2(const void* p, uint64_t& w0, uint64_t& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}

template <typename TV, int W>
__global__ void __launch_bounds__(128) fused_ll_ar_opt_kernel(FusedARArgs a) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  const int world = W > 0 ? W : a.world;
  const int me = a.rank;
  const int64_t npair = (a.end - a.start) / 2;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t par = (int64_t)(epoch & 1u) * (world - 1);
  const float* grad = reinterpret_cast<const float*>(a.peer_grads[me]) + a.start;
  // 1. send
  for (int64_t i = tid; i < npair; i += stride) {
    const float2 g = reinterpret_cast<const float2*>(grad)[i];
    for (int d = 1; d < world; ++d) {
      const int k = (me + d) % world;
      const int slot = (me - k - 1 + world) % world;
      uint64_t* dst = reinterpret_cast<uint64_t*>(a.peer_ll[k]) + (par + slot) * a.ll_cap + a.ll_off + 2 * i;
      st_ll2(dst, g.x, g.y, epoch);
    }
  }
  // 2. receive, reduce in rank order, update
  const OptimHyper h = *a.hyper;
  const float gs = a.scale * h.grad_scale;
  const uint64_t* ll = reinterpret_cast<const uint64_t*>(a.my_ll);
  bool alive = true;
  for (int64_t i = tid; i < npair; i += stride) {
    const float2 own = reinterpret_cast<const float2*>(grad)[i];
    float s0 = 0.f, s1 = 0.f;
    for (int r = 0; r < world; ++r) {
      if (r == me) {
        s0 += own.x;
        s1 += own.y;
        continue;
      }
      const uint64_t* src = ll + (par + (r - me - 1 + world) % world) * a.ll_cap + a.ll_off + 2 * i;
      uint64_t w0 = 0, w1 = 0;
      if (alive) {
        ld_ll2(src, w0, w1);
        if ((uint32_t)(w0 >> 32) != epoch || (uint32_t)(w1 >> 32) != epoch) {
          const uint64_t t0 = gtimer();
          uint32_t it = 0;
          while (true) {
            ld_ll2(src, w0, w1);
            if ((uint32_t)(w0 >> 32) == epoch && (uint32_t)(w1 >> 32) == epoch) break;
            if ((++it & 63u) == 0 && gtimer() - t0 > a.budget_ns) {
              atomicCAS(a.err, 0u, (uint32_t)DLVK_ERR_PEER_TIMEOUT);
              alive = false;
              w0 = w1 = 0;
              break;
            }
          }
        }
      }
      s0 += __uint_as_float((uint32_t)w0);
      s1 += __uint_as_float((uint32_t)w1);
    }
    if (!alive) continue;
    const int64_t e0 = a.start + 2 * i;
    float w[2] = {a.master[e0], a.master[e0 + 1]};
    float m2[2] = {0.f, 0.f}, v2[2] = {0.f, 0.f};
    if (a.m) {
      m2[0] = a.m[e0];
      m2[1] = a.m[e0 + 1];
    }
    if (a.v) {
      v2[0] = a.v[e0];
      v2[1] = a.v[e0 + 1];
    }
    opt_apply(a.kind, h, w[0], s0 * gs, m2[0], v2[0]);
    opt_apply(a.kind, h, w[1], s1 * gs, m2[1], v2[1]);
    a.master[e0] = w[0];
    a.master[e0 + 1] = w[1];
    if (a.m) {
      a.m[e0] = m2[0];
      a.m[e0 + 1] = m2[1];
    }
    if (a.v) {
      a.v[e0] = v2[0];
      a.v[e0 + 1] = v2[1];
    }
    if (!a.values_are_master) {
      TV* out = reinterpret_cast<TV*>(a.peer_values[me]) + e0;
      out[0] = from_f32<TV>(w[0]);
      out[1] = from_f32<TV>(w[1]);
    }
  }
}

template <typename TG, typename TV>
void launch_push(const FusedARArgs& a, int grid, cudaStream_t s) {
  switch (a.world) {
    case 2: fused_push_ar_opt_kernel<TG, TV, 2, 2><<<grid, 256, 0, s>>>(a); break;
    case 4: fused_push_ar_opt_kernel<TG, TV, 4, 2><<<grid, 256, 0, s>>>(a); break;
    case 8: fused_push_ar_opt_kernel<TG, TV, 8, 1><<<grid, 256, 0, s>>>(a); break;
    default: fused_push_ar_opt_kernel<TG, TV, 0, 1><<<grid, 256, 0, s>>>(a); break;
  }
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

void fused_allreduce_optimizer_ll(const FusedARArgs& a, DType value_dt, int ctas, cudaStream_t s) {
  const int64_t n = a.end - a.start;
  if (n <= 0) return;
  DLVK_CHECK(a.world >= 2 && a.world <= 64, "LL all-reduce: world size must be in [2, 64]");
  DLVK_CHECK(a.start % 64 == 0 && n % 64 == 0, "LL all-reduce: bucket must be 64-element aligned");
  DLVK_CHECK(a.peer_ll && a.my_ll && a.ll_off % 2 == 0 && a.ll_off + n <= a.ll_cap, "LL all-reduce: buffer");
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ctas, (n / 2 + 127) / 128));
  auto launch = [&](auto tv) {
    using TV = decltype(tv);
    switch (a.world) {
      case 2: fused_ll_ar_opt_kernel<TV, 2><<<grid, 128, 0, s>>>(a); break;
      case 4: fused_ll_ar_opt_kernel<TV, 4><<<grid, 128, 0, s>>>(a); break;
      case 8: fused_ll_ar_opt_kernel<TV, 8><<<grid, 128, 0, s>>>(a); break;
      default: fused_ll_ar_opt_kernel<TV, 0><<<grid, 128, 0, s>>>(a); break;
    }
  };
  if (value_dt == DType::BF16) launch(__nv_bfloat16{});
  else if (value_dt == DType::F32) launch(float{});
  else throw std::runtime_error("LL all-reduce: unsupported value dtype");
  DLVK_POST_LAUNCH();
}

void fused_allreduce_optimizer_push(const FusedARArgs& a, DType grad_dt, DType value_dt, cudaStream_t s) {
  const int64_t n = a.end - a.start;
  if (n <= 0) return;
  DLVK_CHECK(a.world >= 2 && a.world <= 64, "push all-reduce: world size must be in [2, 64]");
  DLVK_CHECK(a.start % 64 == 0 && n % 64 == 0, "push all-reduce: bucket must be 64-element aligned");
  DLVK_CHECK(a.cbucket >= 0 && a.cbucket < PUSH_MAX_BUCKETS, "push all-reduce: chunk-flag row out of range");
  DLVK_CHECK(a.peer_recv && a.my_recv && a.peer_cflags && a.my_cflags, "push all-reduce: buffers not set");
  const int64_t shard = ((n + a.world - 1) / a.world + 63) / 64 * 64;
  DLVK_CHECK(a.chunk >= 2048 && a.chunk % 1024 == 0, "push all-reduce: bad chunk size");
  DLVK_CHECK(a.recv_off % 64 == 0 && a.recv_off + shard <= a.recv_slot, "push all-reduce: receive slot overflow");
  const int grid = (int)((shard + a.chunk - 1) / a.chunk);
  DLVK_CHECK((int64_t)grid * PUSH_SUB <= PUSH_MAX_CHUNKS, "push all-reduce: too many chunks");
  // One wave: every CTA must be resident at once (CTA c waits on the peers'
  // CTA c only, but a CTA that cannot be scheduled would stall its chunk).
  int dev = 0, sms = 0;
  DLVK_CUDA_CHECK(cudaGetDevice(&dev));
  DLVK_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  DLVK_CHECK(grid <= 2 * sms, "push all-reduce: grid larger than one wave");
  if (grad_dt == DType::F32 && value_dt == DType::BF16) launch_push<float, __nv_bfloat16>(a, grid, s);
  else if (grad_dt == DType::F32 && value_dt == DType::F32) launch_push<float, float>(a, grid, s);
  else if (grad_dt == DType::BF16 && value_dt == DType::BF16) launch_push<__nv_bfloat16, __nv_bfloat16>(a, grid, s);
  else throw std::runtime_error("push all-reduce: unsupported grad/value dtypes");
  DLVK_POST_LAUNCH();
}

void fused_allreduce_optimizer_nvls(const FusedARArgs& a, DType value_dt, int ctas, cudaStream_t s) {
  DLVK_CHECK(a.mc_grads != nullptr && a.mc_values != nullptr, "NVLS all-reduce: multicast addresses missing");
  DLVK_CHECK(a.values_are_master == (value_dt == DType::F32 ? 1 : 0),
             "NVLS all-reduce: fp32 values must be the master copy, bf16 values a mirror");
  DLVK_CHECK((reinterpret_cast<uintptr_t>(a.mc_grads) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.mc_values) & 15) == 0,
             "NVLS all-reduce: multicast addresses must be 16-byte aligned");
  DLVK_CHECK(a.start % 64 == 0 && (a.end - a.start) % 64 == 0,
             "NVLS all-reduce: the range must start and end on 64-element boundaries");
  const int grid = std::max(1, ctas);
  if (value_dt == DType::F32) fused_nvls_ar_opt_kernel<float, 2><<<grid, 128, 0, s>>>(a);
  else fused_nvls_ar_opt_kernel<__nv_bfloat16, 2><<<grid, 128, 0, s>>>(a);
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

// ---------------------------------------------------------------- collectives
// Pull collectives over the staging symmetric buffer (`peer_grads` = every
// rank's staging base): each rank has written its contribution at offset 0
// of its own staging buffer before the launch; after the ready barrier every
// rank reads what it needs straight from the peers' buffers (P2P loads) into
// its local output; the done barrier then frees the staging buffers for
// reuse.  Copies move 16-byte vectors with a byte tail; the reduce-scatter
// sums in rank order (deterministic).
namespace {
enum CollMode : int { COLL_BROADCAST = 0, COLL_ALL_GATHER = 1, COLL_REDUCE_SCATTER = 2 };

__device__ __forceinline__ void copy_bytes(uint8_t* dst, const uint8_t* src, int64_t nbytes, int64_t tid,
                                           int64_t stride) {
  const int64_t nv = nbytes / 16;
  for (int64_t i = tid; i < nv; i += stride)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int64_t i = nv * 16 + tid; i < nbytes; i += stride) dst[i] = src[i];
}

template <typename T>
__global__ void __launch_bounds__(128, 8) p2p_collective_kernel(FusedARArgs a, void* out, int64_t numel, int mode,
                                                                int root) {
  const uint32_t epoch = (uint32_t)(*a.epoch_ptr);
  if (!ready_barrier(a, epoch)) return;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (mode == COLL_BROADCAST) {
    if (a.rank != root)
      copy_bytes(static_cast<uint8_t*>(out), static_cast<const uint8_t*>(a.peer_grads[root]),
                 numel * (int64_t)sizeof(T), tid, stride);
  } else if (mode == COLL_ALL_GATHER) {
    const int64_t nb = numel * (int64_t)sizeof(T);
    for (int r = 0; r < a.world; ++r)  // rank r's block, in place for every rank
      copy_bytes(static_cast<uint8_t*>(out) + r * nb, static_cast<const uint8_t*>(a.peer_grads[r]), nb, tid, stride);
  } else {
    const int64_t chunk = (numel + a.world - 1) / a.world;
    const int64_t lo = min(numel, chunk * a.rank), hi = min(numel, lo + chunk);
    for (int64_t i = lo + tid; i < hi; i += stride) {
      float acc = 0.f;
      for (int r = 0; r < a.world; ++r) acc += to_f32(reinterpret_cast<const T*>(a.peer_grads[r])[i]);
      static_cast<T*>(out)[i - lo] = from_f32<T>(acc);
    }
  }
  done_barrier(a, epoch);
}
}  // namespace

void p2p_collective(const FusedARArgs& a, DType dt, int mode, int root, void* out, int64_t numel, int ctas,
                    cudaStream_t s) {
  DLVK_CHECK(mode >= 0 && mode <= 2 && root >= 0 && root < a.world, "p2p collective: bad mode or root");
  DLVK_CHECK((reinterpret_cast<uintptr_t>(out) & 15) == 0, "p2p collective: output must be 16-byte aligned");
  const int grid = std::max(1, ctas);
  if (dt == DType::F32) p2p_collective_kernel<float><<<grid, 128, 0, s>>>(a, out, numel, mode, root);
  else if (dt == DType::BF16) p2p_collective_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>(a, out, numel, mode, root);
  else throw std::runtime_error("p2p collective: unsupported dtype");
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
