// Bindings of the layer kernels: convolution, pooling, batch/layer norm,
// dropout and embedding.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "bind_common.h"
#include "dlvk/kernels.h"
#include "dlvk/aten_ops.h"

namespace dlvk {
namespace bind {
using namespace ::dlvk::aten;

void f32c(const at::Tensor& t, const char* what) {
  check_cuda(t, what);
  TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous(), "dlvk.image: ", what, " must be contiguous fp32");
}

void register_image(py::module& m) {
  auto im = m.def_submodule("image", "batched image transforms on the device");
  im.def("affine_sample", [](const at::Tensor& x, const at::Tensor& theta, int64_t oh, int64_t ow, int mode,
                             double fill) {
    f32c(x, "x");
    f32c(theta, "theta");
    TORCH_CHECK(x.dim() == 4 && theta.numel() == x.size(0) * 6, "dlvk.image.affine_sample: x [N,C,H,W], theta [N,6]");
    c10::cuda::CUDAGuard g(x.device());
    auto y = at::empty({x.size(0), x.size(1), oh, ow}, x.options());
    image_affine_sample(x.data_ptr<float>(), y.data_ptr<float>(), (int)x.size(0), (int)x.size(1), (int)x.size(2),
                        (int)x.size(3), (int)oh, (int)ow, theta.data_ptr<float>(), mode, (float)fill, stream());
    return y;
  });
  im.def("per_sample_stats", [](const at::Tensor& x, int kind, c10::optional<at::Tensor> params, bool clamp01) {
    f32c(x, "x");
    const float* pp = nullptr;
    if (params.has_value()) {
      f32c(*params, "params");
      TORCH_CHECK(params->numel() == 2 * x.size(0), "dlvk.image.per_sample_stats: params [N,2]");
      pp = params->data_ptr<float>();
    }
    TORCH_CHECK(kind != 0 || pp, "dlvk.image.per_sample_stats: contrast needs params");
    c10::cuda::CUDAGuard g(x.device());
    auto y = at::empty_like(x);
    const int64_t n = x.size(0);
    image_per_sample_stats(x.data_ptr<float>(), y.data_ptr<float>(), n, n ? x.numel() / n : 0, kind, pp, clamp01,
                           stream());
    return y;
  }, py::arg("x"), py::arg("kind"), py::arg("params") = py::none(), py::arg("clamp01") = false);
  im.def("channel_affine", [](const at::Tensor& x, c10::optional<at::Tensor> mean, c10::optional<at::Tensor> inv_std,
                              c10::optional<at::Tensor> sample_add, bool clamp01) {
    f32c(x, "x");
    TORCH_CHECK(x.dim() >= 2, "dlvk.image.channel_affine: x [N,C,...]");
    const int64_t N = x.size(0), C = x.size(1), HW = (N * C) ? x.numel() / (N * C) : 0;
    const float *mp = nullptr, *ip = nullptr, *ap = nullptr;
    if (mean.has_value()) {
      f32c(*mean, "mean");
      TORCH_CHECK(inv_std.has_value() && mean->numel() == C && inv_std->numel() == C, "dlvk.image: mean/inv_std [C]");
      f32c(*inv_std, "inv_std");
      mp = mean->data_ptr<float>();
      ip = inv_std->data_ptr<float>();
    }
    if (sample_add.has_value()) {
      f32c(*sample_add, "sample_add");
      TORCH_CHECK(sample_add->numel() == N, "dlvk.image: sample_add [N]");
      ap = sample_add->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(x.device());
    auto y = at::empty_like(x);
    image_channel_affine(x.data_ptr<float>(), y.data_ptr<float>(), N, (int)C, HW, mp, ip, ap, clamp01, stream());
    return y;
  }, py::arg("x"), py::arg("mean") = py::none(), py::arg("inv_std") = py::none(), py::arg("sample_add") = py::none(),
     py::arg("clamp01") = false);
  im.def("gaussian_noise", [](const at::Tensor& x, double sigma, uint64_t seed, uint32_t stream_id) {
    f32c(x, "x");
    c10::cuda::CUDAGuard g(x.device());
    auto y = at::empty_like(x);
    image_gaussian_noise(x.data_ptr<float>(), y.data_ptr<float>(), x.numel(), (float)sigma, seed, stream_id, stream());
    return y;
  });
}

// A [B, X] row view (unit inner stride): (pointer, row stride).
std::pair<const void*, int64_t> rows_of(const c10::optional<at::Tensor>& t, const char* what, int64_t B) {
  if (!t.has_value()) return {nullptr, 0};
  check_cuda(*t, what);
  TORCH_CHECK(t->dim() == 2 && t->size(0) == B && t->stride(1) == 1, "dlvk.rnn: ", what, " must be a [B, X] row view");
  return {t->data_ptr(), t->stride(0)};
}

void register_rnn(py::module& m) {
  auto r = m.def_submodule("rnn", "recurrent cell kernels");
  r.def("cell_fwd", [](int kind, int64_t H, const at::Tensor& a, c10::optional<at::Tensor> hg,
                       c10::optional<at::Tensor> h_prev, c10::optional<at::Tensor> c_prev, at::Tensor h_out,
                       c10::optional<at::Tensor> h_copy, c10::optional<at::Tensor> c_out,
                       c10::optional<at::Tensor> saved) {
    const int64_t B = a.size(0);
    RnnCellFwd p;
    p.kind = kind;
    p.B = B;
    p.H = (int)H;
    std::tie(p.a, p.lda) = rows_of(a, "a", B);
    std::tie(p.hg, p.ldhg) = rows_of(hg, "hg", B);
    std::tie(p.h_prev, p.ldhp) = rows_of(h_prev, "h_prev", B);
    auto cp = rows_of(c_prev, "c_prev", B);
    p.c_prev = (const float*)cp.first;
    p.ldcp = cp.second;
    auto ho = rows_of(h_out, "h_out", B);
    p.h_out = const_cast<void*>(ho.first);
    p.ldo = ho.second;
    auto hc = rows_of(h_copy, "h_copy", B);
    p.h_copy = const_cast<void*>(hc.first);
    p.ldcopy = hc.second;
    auto co = rows_of(c_out, "c_out", B);
    p.c_out = (float*)co.first;
    p.ldco = co.second;
    auto sv = rows_of(saved, "saved", B);
    p.saved = (float*)sv.first;
    p.lds = sv.second;
    TORCH_CHECK(a.scalar_type() == h_out.scalar_type(), "dlvk.rnn: a and h_out dtype");
    TORCH_CHECK(kind == 0 || p.saved, "dlvk.rnn: saved gates required");
    TORCH_CHECK(kind != 1 || p.c_out, "dlvk.rnn: LSTM needs c_out");
    TORCH_CHECK(kind != 2 || p.hg, "dlvk.rnn: GRU needs hg");
    c10::cuda::CUDAGuard g(a.device());
    rnn_cell_fwd(p, to_dtype(a), stream());
  }, py::arg("kind"), py::arg("H"), py::arg("a"), py::arg("hg"), py::arg("h_prev"), py::arg("c_prev"),
     py::arg("h_out"), py::arg("h_copy"), py::arg("c_out"), py::arg("saved"));
  r.def("cell_bwd", [](int kind, int64_t H, const at::Tensor& dh, c10::optional<at::Tensor> dc_next,
                       c10::optional<at::Tensor> h_t, c10::optional<at::Tensor> h_prev, c10::optional<at::Tensor> c_t,
                       c10::optional<at::Tensor> c_prev, c10::optional<at::Tensor> saved, at::Tensor dA,
                       c10::optional<at::Tensor> dAh, c10::optional<at::Tensor> dc_prev,
                       c10::optional<at::Tensor> dy_prev, c10::optional<at::Tensor> resid) {
    const int64_t B = dh.size(0);
    RnnCellBwd p;
    p.kind = kind;
    p.B = B;
    p.H = (int)H;
    std::tie(p.dh, p.lddh) = rows_of(dh, "dh", B);
    auto dcn = rows_of(dc_next, "dc_next", B);
    p.dc_next = (const float*)dcn.first;
    p.lddcn = dcn.second;
    std::tie(p.h_t, p.ldht) = rows_of(h_t, "h_t", B);
    std::tie(p.h_prev, p.ldhp) = rows_of(h_prev, "h_prev", B);
    auto ct = rows_of(c_t, "c_t", B);
    p.c_t = (const float*)ct.first;
    p.ldct = ct.second;
    auto cp = rows_of(c_prev, "c_prev", B);
    p.c_prev = (const float*)cp.first;
    p.ldcp = cp.second;
    auto sv = rows_of(saved, "saved", B);
    p.saved = (const float*)sv.first;
    p.lds = sv.second;
    auto da = rows_of(dA, "dA", B);
    p.dA = const_cast<void*>(da.first);
    p.ldda = da.second;
    auto dah = rows_of(dAh, "dAh", B);
    p.dAh = const_cast<void*>(dah.first);
    p.lddah = dah.second;
    auto dcp = rows_of(dc_prev, "dc_prev", B);
    p.dc_prev = (float*)dcp.first;
    p.lddcp = dcp.second;
    std::tie(p.dy_prev, p.lddyp) = rows_of(dy_prev, "dy_prev", B);
    auto rs = rows_of(resid, "resid", B);
    p.resid = const_cast<void*>(rs.first);
    p.ldres = rs.second;
    TORCH_CHECK(kind != 0 || p.h_t, "dlvk.rnn: RNN bwd needs h_t");
    TORCH_CHECK(kind != 1 || (p.c_t && p.saved && p.dc_prev), "dlvk.rnn: LSTM bwd needs c_t, saved, dc_prev");
    TORCH_CHECK(kind != 2 || (p.saved && p.dAh), "dlvk.rnn: GRU bwd needs saved, dAh");
    c10::cuda::CUDAGuard g(dh.device());
    rnn_cell_bwd(p, to_dtype(dh), stream());
  }, py::arg("kind"), py::arg("H"), py::arg("dh"), py::arg("dc_next"), py::arg("h_t"), py::arg("h_prev"),
     py::arg("c_t"), py::arg("c_prev"), py::arg("saved"), py::arg("dA"), py::arg("dAh"), py::arg("dc_prev"),
     py::arg("dy_prev"), py::arg("resid"));
}

void bf16c(const at::Tensor& t, const char* what) {
  check_cuda(t, what);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "dlvk.flash_attn: ", what,
              " must be contiguous bf16");
}

void register_attention(py::module& m) {
  m.def("flash_attn_supported", [](int64_t B, int64_t S, int64_t H, int64_t D, const at::Tensor& qkv) {
    return qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() &&
           flash_attention_supported(B, S, H, D, qkv.data_ptr());
  });
  m.def("flash_attn_fwd", [](const at::Tensor& qkv, int64_t B, int64_t S, int64_t H, double scale,
                             int64_t max_ctas) {
    bf16c(qkv, "qkv");
    TORCH_CHECK(qkv.numel() == B * S * 3 * H * 64, "dlvk.flash_attn_fwd: qkv must be [B, S, 3*H*64]");
    c10::cuda::CUDAGuard g(qkv.device());
    auto out = at::empty({B, S, H * 64}, qkv.options());
    auto lse = at::empty({B, H, S}, qkv.options().dtype(at::kFloat));
    flash_attention_fwd(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), (int)B, (int)S,
                        (int)H, (float)scale, stream(), device_error_word(), (int)max_ctas);
    return py::make_tuple(out, lse);
  }, py::arg("qkv"), py::arg("B"), py::arg("S"), py::arg("H"), py::arg("scale"), py::arg("max_ctas") = 0);
  m.def("flash_attn_bwd", [](const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout,
                             const at::Tensor& lse, int64_t B, int64_t S, int64_t H, double scale, int64_t max_ctas) {
    bf16c(qkv, "qkv");
    bf16c(out, "out");
    bf16c(dout, "dout");
    check_cuda(lse, "lse");
    TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * S && lse.is_contiguous(),
                "dlvk.flash_attn_bwd: lse [B, H, S] fp32");
    TORCH_CHECK(out.numel() == B * S * H * 64 && dout.numel() == out.numel(), "dlvk.flash_attn_bwd: out/dout shape");
    c10::cuda::CUDAGuard g(qkv.device());
    auto dqkv = at::empty({B, S, 3 * H * 64}, qkv.options());
    auto delta = at::empty({B, H, S}, lse.options());
    auto acc = at::empty({B * S, H * 64}, lse.options());
    flash_attention_bwd(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), lse.data_ptr<float>(),
                        delta.data_ptr<float>(), acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
                        (int)B, (int)S, (int)H, (float)scale, stream(), device_error_word(), (int)max_ctas);
    return dqkv;
  }, py::arg("qkv"), py::arg("out"), py::arg("dout"), py::arg("lse"), py::arg("B"), py::arg("S"), py::arg("H"),
     py::arg("scale"), py::arg("max_ctas") = 0);
}

void register_nn(py::module& m) {
  register_image(m);
  register_attention(m);
  register_rnn(m);
  m.def("quantize_rows", &quantize_rows_op);
  m.def("gemm_i8", &gemm_i8_op, py::arg("qa"), py::arg("qbt"), py::arg("sa"), py::arg("sb"),
        py::arg("bias") = py::none(), py::arg("act") = 0, py::arg("out_dtype") = py::none(),
        py::arg("force_path") = 0);
  m.def("conv2d_fwd", &conv2d_fwd_op, py::arg("x"), py::arg("w"), py::arg("bias") = py::none(), py::arg("stride") = 1,
        py::arg("pad") = 0, py::arg("relu") = false);
  m.def("conv2d_dgrad", &conv2d_dgrad_op, py::arg("gy"), py::arg("w"), py::arg("xshape"), py::arg("stride") = 1,
        py::arg("pad") = 0, py::arg("relu_src") = py::none());
  m.def("conv2d_wgrad", &conv2d_wgrad_op, py::arg("x"), py::arg("gy"), py::arg("dw"), py::arg("db") = py::none(),
        py::arg("stride") = 1, py::arg("pad") = 0, py::arg("accumulate") = false);
  m.def("conv_tc_set_mode", &conv_tc_set_mode, "0 auto, 1 tensor-core implicit GEMM whenever supported, 2 never");
  m.def("conv_tc_get_mode", &conv_tc_get_mode);
  m.def("maxpool_fwd", &maxpool_fwd_op);
  m.def("maxpool_bwd", &maxpool_bwd_op);
  m.def("avgpool_fwd", &avgpool_fwd_op);
  m.def("avgpool_bwd", &avgpool_bwd_op);
  m.def("batchnorm_fwd", &batchnorm_fwd_op, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("run_mean"),
        py::arg("run_var"), py::arg("momentum") = 0.1, py::arg("eps") = 1e-5, py::arg("training") = true,
        py::arg("relu") = false, py::arg("p") = 0.0, py::arg("stream_id") = 0, py::arg("seed") = 0,
        py::arg("step") = 0, py::arg("step_t") = py::none());
  m.def("batchnorm_bwd", &batchnorm_bwd_op, py::arg("x"), py::arg("dy"), py::arg("mean"), py::arg("rstd"),
        py::arg("gamma"), py::arg("beta"), py::arg("dgamma"), py::arg("dbeta"), py::arg("accumulate") = false,
        py::arg("relu") = false, py::arg("p") = 0.0, py::arg("stream_id") = 0, py::arg("seed") = 0,
        py::arg("step") = 0, py::arg("step_t") = py::none());
  m.def("layernorm_fwd", &layernorm_fwd_op, py::arg("x"), py::arg("gamma"), py::arg("beta"), py::arg("eps") = 1e-5);
  m.def("layernorm_bwd", &layernorm_bwd_op, py::arg("x"), py::arg("gamma"), py::arg("mean"), py::arg("rstd"),
        py::arg("dy"), py::arg("dgamma"), py::arg("dbeta"), py::arg("accumulate") = false,
        py::arg("dres") = py::none(), py::arg("dres_colsum") = py::none(), py::arg("dres_colsum_accumulate") = false);
  m.def("dropout", &dropout_op, py::arg("x"), py::arg("p"), py::arg("stream_id") = 0, py::arg("seed") = 0,
        py::arg("step") = 0, py::arg("step_t") = py::none());
  m.def("embedding_fwd", &embedding_fwd_op);
  m.def("embedding_bwd", &embedding_bwd_op);
}

}  // namespace bind
}  // namespace dlvk
