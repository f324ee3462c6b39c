// Recurrent cell kernels (RNN-tanh, LSTM, GRU), forward and backward.
//
// Reference: RNN/LSTM/GRU layers of include/dlvk/layers/recurrent_layers.h:
// 18-200 (weights [G*H, I] and [G*H, H], gate order LSTM i,f,g,o with the
// forget-gate bias initialised to 1, src/layers/recurrent_layers.cpp:
// 195-215; GRU r,z,n).  The reference's forward returns zeros and its
// backward an empty tensor (recurrent_layers.cpp:19-56); this is the
// working version.
//
// Per time step the host runs ONE tensor-core GEMM (h_{t-1} W_hh^T, with the
// precomputed input projection x_t W_ih^T + b added in the epilogue for
// RNN/LSTM) and ONE of these element-wise cell kernels; backward runs the
// cell-backward kernel and one GEMM for dh_{t-1} (adding dY_{t-1} in the
// epilogue), and the weight gradients are two large GEMMs over all steps
// after the loop.  Every buffer is addressed as rows of a batch with its own
// row stride, so time slices of [B, T, *] tensors and the halves of a
// bidirectional output are read and written in place.
//
// Saved state is fp32: LSTM gates (i, f, g, o) and cell states, GRU
// (r, z, n, hn) where hn = h_{t-1} W_hn^T + b_hn.
#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace {

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

template <typename T>
__global__ void cell_fwd_kernel(int kind, int64_t B, int H, const T* __restrict__ a, int64_t lda,
                                const T* __restrict__ hg, int64_t ldhg, const T* __restrict__ h_prev, int64_t ldhp,
                                const float* __restrict__ c_prev, int64_t ldcp, T* __restrict__ h_out, int64_t ldo,
                                T* __restrict__ h_copy, int64_t ldcopy, float* __restrict__ c_out, int64_t ldco,
                                float* __restrict__ saved, int64_t lds) {
  const int64_t total = B * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / H;
    const int j = (int)(i % H);
    const T* ar = a + b * lda;
    float h;
    if (kind == 0) {
      h = tanhf(to_f32(ar[j]));
    } else if (kind == 1) {
      const float ig = sigm(to_f32(ar[j])), fg = sigm(to_f32(ar[H + j]));
      const float gg = tanhf(to_f32(ar[2 * H + j])), og = sigm(to_f32(ar[3 * H + j]));
      const float cp = c_prev ? c_prev[b * ldcp + j] : 0.f;
      const float c = fg * cp + ig * gg;
      h = og * tanhf(c);
      c_out[b * ldco + j] = c;
      float* sv = saved + b * lds;
      sv[j] = ig;
      sv[H + j] = fg;
      sv[2 * H + j] = gg;
      sv[3 * H + j] = og;
    } else {
      const T* hr = hg + b * ldhg;
      const float r = sigm(to_f32(ar[j]) + to_f32(hr[j]));
      const float z = sigm(to_f32(ar[H + j]) + to_f32(hr[H + j]));
      const float hn = to_f32(hr[2 * H + j]);
      const float n = tanhf(to_f32(ar[2 * H + j]) + r * hn);
      const float hp = h_prev ? to_f32(h_prev[b * ldhp + j]) : 0.f;
      h = (1.f - z) * n + z * hp;
      float* sv = saved + b * lds;
      sv[j] = r;
      sv[H + j] = z;
      sv[2 * H + j] = n;
      sv[3 * H + j] = hn;
    }
    const T hv = from_f32<T>(h);
    h_out[b * ldo + j] = hv;
    if (h_copy) h_copy[b * ldcopy + j] = hv;
  }
}

// dh: total gradient of h_t.  Writes dA (grad of the input-side
// pre-activations, [B, G*H] rows), for GRU also dAh (hidden-side
// pre-activations) and resid = dh * z + dy_prev (the non-GEMM part of
// dh_{t-1}); for LSTM dc_prev.
template <typename T>
__global__ void cell_bwd_kernel(int kind, int64_t B, int H, const T* __restrict__ dh, int64_t lddh,
                                const float* __restrict__ dc_next, int64_t lddcn, const T* __restrict__ h_t,
                                int64_t ldht, const T* __restrict__ h_prev, int64_t ldhp,
                                const float* __restrict__ c_t, int64_t ldct, const float* __restrict__ c_prev,
                                int64_t ldcp, const float* __restrict__ saved, int64_t lds, T* __restrict__ dA,
                                int64_t ldda, T* __restrict__ dAh, int64_t lddah, float* __restrict__ dc_prev,
                                int64_t lddcp, const T* __restrict__ dy_prev, int64_t lddyp, T* __restrict__ resid,
                                int64_t ldres) {
  const int64_t total = B * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / H;
    const int j = (int)(i % H);
    const float g = to_f32(dh[b * lddh + j]);
    T* da = dA + b * ldda;
    if (kind == 0) {
      const float h = to_f32(h_t[b * ldht + j]);
      da[j] = from_f32<T>(g * (1.f - h * h));
    } else if (kind == 1) {
      const float* sv = saved + b * lds;
      const float ig = sv[j], fg = sv[H + j], gg = sv[2 * H + j], og = sv[3 * H + j];
      const float c = c_t[b * ldct + j];
      const float tc = tanhf(c);
      float dc = g * og * (1.f - tc * tc);
      if (dc_next) dc += dc_next[b * lddcn + j];
      const float cp = c_prev ? c_prev[b * ldcp + j] : 0.f;
      da[j] = from_f32<T>(dc * gg * ig * (1.f - ig));
      da[H + j] = from_f32<T>(dc * cp * fg * (1.f - fg));
      da[2 * H + j] = from_f32<T>(dc * ig * (1.f - gg * gg));
      da[3 * H + j] = from_f32<T>(g * tc * og * (1.f - og));
      dc_prev[b * lddcp + j] = dc * fg;
    } else {
      const float* sv = saved + b * lds;
      const float r = sv[j], z = sv[H + j], n = sv[2 * H + j], hn = sv[3 * H + j];
      const float hp = h_prev ? to_f32(h_prev[b * ldhp + j]) : 0.f;
      const float dn = g * (1.f - z) * (1.f - n * n);
      const float dz = g * (hp - n) * z * (1.f - z);
      const float dr = dn * hn * r * (1.f - r);
      da[j] = from_f32<T>(dr);
      da[H + j] = from_f32<T>(dz);
      da[2 * H + j] = from_f32<T>(dn);
      T* dah = dAh + b * lddah;
      dah[j] = from_f32<T>(dr);
      dah[H + j] = from_f32<T>(dz);
      dah[2 * H + j] = from_f32<T>(dn * r);
      if (resid) {
        float rv = g * z;
        if (dy_prev) rv += to_f32(dy_prev[b * lddyp + j]);
        resid[b * ldres + j] = from_f32<T>(rv);
      }
    }
  }
}

int grid_for_cells(int64_t n) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8)); }

}  // namespace

void rnn_cell_fwd(const RnnCellFwd& p, DType dt, cudaStream_t s) {
  const int64_t n = p.B * p.H;
  if (n == 0) return;
#define DLVK_CELL_FWD(T)                                                                                           \
  cell_fwd_kernel<T><<<grid_for_cells(n), 256, 0, s>>>(                                                            \
      p.kind, p.B, p.H, (const T*)p.a, p.lda, (const T*)p.hg, p.ldhg, (const T*)p.h_prev, p.ldhp, p.c_prev, p.ldcp, \
      (T*)p.h_out, p.ldo, (T*)p.h_copy, p.ldcopy, p.c_out, p.ldco, p.saved, p.lds)
  if (dt == DType::F32)
    DLVK_CELL_FWD(float);
  else if (dt == DType::BF16)
    DLVK_CELL_FWD(__nv_bfloat16);
  else
    throw std::runtime_error("dlvk::rnn_cell_fwd: unsupported dtype");
#undef DLVK_CELL_FWD
  DLVK_POST_LAUNCH();
}

void rnn_cell_bwd(const RnnCellBwd& p, DType dt, cudaStream_t s) {
  const int64_t n = p.B * p.H;
  if (n == 0) return;
#define DLVK_CELL_BWD(T)                                                                                            \
  cell_bwd_kernel<T><<<grid_for_cells(n), 256, 0, s>>>(                                                             \
      p.kind, p.B, p.H, (const T*)p.dh, p.lddh, p.dc_next, p.lddcn, (const T*)p.h_t, p.ldht, (const T*)p.h_prev,    \
      p.ldhp, p.c_t, p.ldct, p.c_prev, p.ldcp, p.saved, p.lds, (T*)p.dA, p.ldda, (T*)p.dAh, p.lddah, p.dc_prev,     \
      p.lddcp, (const T*)p.dy_prev, p.lddyp, (T*)p.resid, p.ldres)
  if (dt == DType::F32)
    DLVK_CELL_BWD(float);
  else if (dt == DType::BF16)
    DLVK_CELL_BWD(__nv_bfloat16);
  else
    throw std::runtime_error("dlvk::rnn_cell_bwd: unsupported dtype");
#undef DLVK_CELL_BWD
  DLVK_POST_LAUNCH();
}

}  // namespace dlvk
