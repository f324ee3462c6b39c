// Bindings of the layer kernels: convolution, pooling, batch/layer norm,
// dropout and embedding.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "bind_common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace bind {
namespace {

const float* optf(const c10::optional<at::Tensor>& t) {
  if (!t.has_value()) return nullptr;
  TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->is_cuda(), "dlvk: expected f32 CUDA tensor");
  return t->data_ptr<float>();
}
float* optfm(const c10::optional<at::Tensor>& t) { return const_cast<float*>(optf(t)); }

ConvDesc conv_desc(const at::Tensor& x, const at::Tensor& w, int64_t stride, int64_t pad) {
  TORCH_CHECK(x.dim() == 4 && w.dim() == 4 && x.size(1) == w.size(1), "dlvk.conv2d: NCHW input, [Cout,Cin,KH,KW] weight");
  ConvDesc d;
  d.N = (int)x.size(0);
  d.Cin = (int)x.size(1);
  d.H = (int)x.size(2);
  d.W = (int)x.size(3);
  d.Cout = (int)w.size(0);
  d.KH = (int)w.size(2);
  d.KW = (int)w.size(3);
  d.stride = (int)stride;
  d.pad = (int)pad;
  d.Ho = (d.H + 2 * d.pad - d.KH) / d.stride + 1;
  d.Wo = (d.W + 2 * d.pad - d.KW) / d.stride + 1;
  return d;
}

DropoutDesc drop_desc(double p, int64_t stream_id, int64_t seed, int64_t step, const c10::optional<at::Tensor>& step_t) {
  DropoutDesc dd;
  dd.p = (float)p;
  dd.stream = (uint32_t)stream_id;
  dd.seed = (uint64_t)seed;
  dd.step = (uint32_t)step;
  if (step_t.has_value()) {
    TORCH_CHECK(step_t->scalar_type() == at::kLong && step_t->is_cuda(), "dlvk: step counter must be int64 CUDA");
    dd.step_ptr = step_t->data_ptr<int64_t>();
  }
  return dd;
}

// NCHW -> NHWC copy of a bf16 activation (one batched 2-D transpose).
at::Tensor to_nhwc(const at::Tensor& x) {
  auto y = at::empty({x.size(0), x.size(2), x.size(3), x.size(1)}, x.options());
  transpose2d(DType::BF16, x.data_ptr(), y.data_ptr(), x.size(0), x.size(1), x.size(2) * x.size(3), stream());
  return y;
}

at::Tensor pack_conv_weights(const at::Tensor& w, const ConvDesc& d, bool dgrad) {
  const int64_t rows = dgrad ? d.Cin : d.Cout;
  const int64_t cols = conv_pack_cols((int64_t)d.KH * d.KW * (dgrad ? d.Cout : d.Cin));
  auto wp = at::empty({rows, cols}, w.options().dtype(at::kBFloat16));
  conv_pack_weights(to_dtype(w), w.data_ptr(), reinterpret_cast<__nv_bfloat16*>(wp.data_ptr()), d, dgrad, stream());
  return wp;
}

const __nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }

at::Tensor conv2d_fwd_op(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias, int64_t stride,
                         int64_t pad, bool relu) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), wc = w.contiguous().to(x.scalar_type());
  auto d = conv_desc(xc, wc, stride, pad);
  auto y = at::empty({d.N, d.Cout, d.Ho, d.Wo}, xc.options());
  if (conv2d_tc_supported(to_dtype(xc), d)) {
    auto xn = to_nhwc(xc);
    auto wp = pack_conv_weights(wc, d, false);
    conv2d_igemm(bf(xn), bf(wp), d, false, optf(bias), relu, nullptr, y.data_ptr(), false, stream());
    return y;
  }
  conv2d_fwd(to_dtype(xc), xc.data_ptr(), wc.data_ptr(), optf(bias), y.data_ptr(), d, relu, stream());
  return y;
}

at::Tensor conv2d_dgrad_op(const at::Tensor& gy, const at::Tensor& w, std::vector<int64_t> xshape, int64_t stride,
                           int64_t pad, c10::optional<at::Tensor> relu_src) {
  check_cuda(gy, "gy");
  c10::cuda::CUDAGuard g(gy.device());
  auto gc = gy.contiguous(), wc = w.contiguous().to(gy.scalar_type());
  auto dx = at::empty(xshape, gc.options());
  auto d = conv_desc(dx, wc, stride, pad);
  TORCH_CHECK(gc.size(2) == d.Ho && gc.size(3) == d.Wo, "dlvk.conv2d_dgrad: grad shape");
  const void* rs = nullptr;
  at::Tensor rsc;
  if (relu_src.has_value()) {
    rsc = relu_src->contiguous();
    TORCH_CHECK(rsc.scalar_type() == gc.scalar_type() && rsc.numel() == dx.numel(), "dlvk.conv2d_dgrad: relu_src");
    rs = rsc.data_ptr();
  }
  if (conv2d_tc_supported(to_dtype(gc), d)) {
    auto gn = to_nhwc(gc);
    auto wp = pack_conv_weights(wc, d, true);
    conv2d_igemm(bf(gn), bf(wp), d, true, nullptr, false, rs, dx.data_ptr(), false, stream());
    return dx;
  }
  conv2d_dgrad(to_dtype(gc), gc.data_ptr(), wc.data_ptr(), dx.data_ptr(), rs, d, stream());
  return dx;
}

void conv2d_wgrad_op(const at::Tensor& x, const at::Tensor& gy, const at::Tensor& dw, c10::optional<at::Tensor> db,
                     int64_t stride, int64_t pad, bool accumulate) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), gc = gy.contiguous().to(x.scalar_type());
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous(), "dlvk.conv2d_wgrad: f32 contiguous dw");
  auto d = conv_desc(xc, dw, stride, pad);
  if (conv2d_tc_supported(to_dtype(xc), d)) {
    TORCH_CHECK(gc.size(2) == d.Ho && gc.size(3) == d.Wo, "dlvk.conv2d_wgrad: grad shape");
    auto xn = to_nhwc(xc);
    auto gn = to_nhwc(gc);
    auto ws = at::empty({conv2d_wgrad_tc_ws_floats(d)}, xc.options().dtype(at::kFloat));
    conv2d_wgrad_tc(bf(xn), bf(gn), d, ws.data_ptr<float>(), dw.data_ptr<float>(), accumulate, stream());
    if (db.has_value()) {
      const int64_t P = (int64_t)d.N * d.Ho * d.Wo;
      auto cs = at::empty({std::max<int64_t>(1, colsum_scratch_floats(P, d.Cout))}, ws.options());
      colsum(DType::BF16, DType::F32, gn.data_ptr(), P, d.Cout, 1.f, db->data_ptr<float>(), accumulate,
             cs.data_ptr<float>(), stream());
    }
    return;
  }
  auto scratch = at::empty({conv2d_wgrad_scratch_floats(d)}, xc.options().dtype(at::kFloat));
  conv2d_wgrad(to_dtype(xc), xc.data_ptr(), gc.data_ptr(), dw.data_ptr<float>(), optfm(db), accumulate, d,
               scratch.data_ptr<float>(), stream());
}

std::vector<at::Tensor> maxpool_fwd_op(const at::Tensor& x, int64_t k, int64_t stride) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t N = xc.size(0), C = xc.size(1), H = xc.size(2), W = xc.size(3);
  const int64_t Ho = (H - k) / stride + 1, Wo = (W - k) / stride + 1;
  auto y = at::empty({N, C, Ho, Wo}, xc.options());
  auto idx = at::empty({N, C, Ho, Wo}, xc.options().dtype(at::kInt));
  maxpool2d_fwd(to_dtype(xc), xc.data_ptr(), y.data_ptr(), idx.data_ptr<int32_t>(), N * C, (int)H, (int)W, (int)k,
                (int)stride, stream());
  return {y, idx};
}

at::Tensor maxpool_bwd_op(const at::Tensor& gy, const at::Tensor& idx, int64_t H, int64_t W, int64_t k, int64_t stride) {
  check_cuda(gy, "gy");
  c10::cuda::CUDAGuard g(gy.device());
  auto gc = gy.contiguous();
  auto dx = at::empty({gc.size(0), gc.size(1), H, W}, gc.options());
  maxpool2d_bwd(to_dtype(gc), gc.data_ptr(), idx.data_ptr<int32_t>(), dx.data_ptr(), gc.size(0) * gc.size(1), (int)H,
                (int)W, (int)k, (int)stride, stream());
  return dx;
}

at::Tensor avgpool_fwd_op(const at::Tensor& x, int64_t k, int64_t stride, int64_t pad) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t N = xc.size(0), C = xc.size(1), H = xc.size(2), W = xc.size(3);
  auto y = at::empty({N, C, (H + 2 * pad - k) / stride + 1, (W + 2 * pad - k) / stride + 1}, xc.options());
  avgpool2d_fwd(to_dtype(xc), xc.data_ptr(), y.data_ptr(), N * C, (int)H, (int)W, (int)k, (int)stride, (int)pad,
                stream());
  return y;
}

at::Tensor avgpool_bwd_op(const at::Tensor& gy, int64_t H, int64_t W, int64_t k, int64_t stride, int64_t pad) {
  check_cuda(gy, "gy");
  c10::cuda::CUDAGuard g(gy.device());
  auto gc = gy.contiguous();
  auto dx = at::empty({gc.size(0), gc.size(1), H, W}, gc.options());
  avgpool2d_bwd(to_dtype(gc), gc.data_ptr(), dx.data_ptr(), gc.size(0) * gc.size(1), (int)H, (int)W, (int)k,
                (int)stride, (int)pad, stream());
  return dx;
}

// Returns (y, mean, rstd).  x is [N, C] or [N, C, *spatial].
std::vector<at::Tensor> batchnorm_fwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma,
                                         c10::optional<at::Tensor> beta, c10::optional<at::Tensor> run_mean,
                                         c10::optional<at::Tensor> run_var, double momentum, double eps,
                                         bool training, bool relu, double p, int64_t stream_id, int64_t seed,
                                         int64_t step, c10::optional<at::Tensor> step_t) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int N = (int)xc.size(0), C = (int)xc.size(1);
  const int S = (int)(xc.numel() / std::max<int64_t>(1, (int64_t)N * C));
  auto y = at::empty_like(xc);
  at::Tensor mean, rstd;
  if (training) {
    mean = at::empty({C}, xc.options().dtype(at::kFloat));
    rstd = at::empty({C}, xc.options().dtype(at::kFloat));
  } else {
    TORCH_CHECK(run_mean.has_value() && run_var.has_value(), "dlvk.batchnorm: eval needs running stats");
    mean = *run_mean;
    rstd = at::rsqrt(*run_var + eps);  // tiny [C] vector
  }
  auto dd = drop_desc(training ? p : 0.0, stream_id, seed, step, step_t);
  auto scratch = at::empty({batchnorm_scratch_floats(N, C, S)}, xc.options().dtype(at::kFloat));
  batchnorm_fwd(to_dtype(xc), xc.data_ptr(), optf(gamma), optf(beta), y.data_ptr(), mean.data_ptr<float>(),
                rstd.data_ptr<float>(), training ? optfm(run_mean) : nullptr, training ? optfm(run_var) : nullptr, N,
                C, S, (float)momentum, (float)eps, training, relu, dd, scratch.data_ptr<float>(), stream());
  return {y, mean, rstd};
}

at::Tensor batchnorm_bwd_op(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& mean, const at::Tensor& rstd,
                            c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> beta,
                            c10::optional<at::Tensor> dgamma, c10::optional<at::Tensor> dbeta, bool accumulate,
                            bool relu, double p, int64_t stream_id, int64_t seed, int64_t step,
                            c10::optional<at::Tensor> step_t) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), dyc = dy.contiguous();
  const int N = (int)xc.size(0), C = (int)xc.size(1);
  const int S = (int)(xc.numel() / std::max<int64_t>(1, (int64_t)N * C));
  auto dx = at::empty_like(xc);
  auto scratch = at::empty({batchnorm_scratch_floats(N, C, S)}, xc.options().dtype(at::kFloat));
  auto dd = drop_desc(p, stream_id, seed, step, step_t);
  batchnorm_bwd(to_dtype(xc), xc.data_ptr(), dyc.data_ptr(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                optf(gamma), optf(beta), dx.data_ptr(), optfm(dgamma), optfm(dbeta), accumulate, N, C, S, relu, dd,
                scratch.data_ptr<float>(), stream());
  return dx;
}

std::vector<at::Tensor> layernorm_fwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma,
                                         c10::optional<at::Tensor> beta, double eps) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t D = xc.size(-1), R = xc.numel() / std::max<int64_t>(D, 1);
  auto y = at::empty_like(xc);
  auto mean = at::empty({R}, xc.options().dtype(at::kFloat));
  auto rstd = at::empty({R}, xc.options().dtype(at::kFloat));
  layernorm_fwd(to_dtype(xc), xc.data_ptr(), optf(gamma), optf(beta), y.data_ptr(), mean.data_ptr<float>(),
                rstd.data_ptr<float>(), R, (int)D, (float)eps, stream());
  return {y, mean, rstd};
}

at::Tensor layernorm_bwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma, const at::Tensor& mean,
                            const at::Tensor& rstd, const at::Tensor& dy, c10::optional<at::Tensor> dgamma,
                            c10::optional<at::Tensor> dbeta, bool accumulate, c10::optional<at::Tensor> dres) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), dyc = dy.contiguous();
  const int64_t D = xc.size(-1), R = xc.numel() / std::max<int64_t>(D, 1);
  auto dx = at::empty_like(xc);
  auto scratch = at::empty({layernorm_bwd_scratch_floats(R, (int)D)}, xc.options().dtype(at::kFloat));
  at::Tensor drc;
  if (dres.has_value()) {
    drc = dres->contiguous();
    TORCH_CHECK(drc.scalar_type() == xc.scalar_type() && drc.numel() == xc.numel(), "dlvk.layernorm_bwd: dres");
  }
  layernorm_bwd(to_dtype(xc), xc.data_ptr(), optf(gamma), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                dyc.data_ptr(), dx.data_ptr(), optfm(dgamma), optfm(dbeta), accumulate, R, (int)D,
                scratch.data_ptr<float>(), stream(), dres.has_value() ? drc.data_ptr() : nullptr);
  return dx;
}

at::Tensor dropout_op(const at::Tensor& x, double p, int64_t stream_id, int64_t seed, int64_t step,
                      c10::optional<at::Tensor> step_t) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  auto y = at::empty_like(xc);
  dropout(to_dtype(xc), xc.data_ptr(), y.data_ptr(), xc.numel(), drop_desc(p, stream_id, seed, step, step_t), stream());
  return y;
}

at::Tensor embedding_fwd_op(const at::Tensor& ids, const at::Tensor& table) {
  check_cuda(table, "table");
  c10::cuda::CUDAGuard g(table.device());
  TORCH_CHECK(ids.scalar_type() == at::kInt, "dlvk.embedding: int32 ids");
  auto idc = ids.contiguous();
  auto tc = table.contiguous();
  std::vector<int64_t> shp(idc.sizes().begin(), idc.sizes().end());
  shp.push_back(tc.size(1));
  auto out = at::empty(shp, tc.options());
  embedding_fwd(to_dtype(tc), idc.data_ptr<int32_t>(), tc.data_ptr(), out.data_ptr(), idc.numel(), tc.size(0),
                (int)tc.size(1), stream());
  return out;
}

void embedding_bwd_op(const at::Tensor& ids, const at::Tensor& dy, const at::Tensor& dtable) {
  check_cuda(dy, "dy");
  c10::cuda::CUDAGuard g(dy.device());
  TORCH_CHECK(dtable.scalar_type() == at::kFloat && dtable.is_contiguous(), "dlvk.embedding_bwd: f32 table grad");
  auto idc = ids.contiguous();
  auto dyc = dy.contiguous();
  embedding_bwd(to_dtype(dyc), idc.data_ptr<int32_t>(), dyc.data_ptr(), dtable.data_ptr<float>(), idc.numel(),
                dtable.size(0), (int)dtable.size(1), stream());
}

std::vector<at::Tensor> quantize_rows_op(const at::Tensor& x) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t cols = xc.size(-1), rows = xc.numel() / std::max<int64_t>(cols, 1);
  auto q = at::empty({rows, cols}, xc.options().dtype(at::kChar));
  auto sc = at::empty({rows}, xc.options().dtype(at::kFloat));
  quantize_rows_int8(to_dtype(xc), xc.data_ptr(), rows, cols, cols, q.data_ptr<int8_t>(), cols, sc.data_ptr<float>(),
                     stream());
  return {q, sc};
}

// y = act(qa @ qbt^T * sa[:, None] * sb[None, :] + bias)
at::Tensor gemm_i8_op(const at::Tensor& qa, const at::Tensor& qbt, const at::Tensor& sa, const at::Tensor& sb,
                      c10::optional<at::Tensor> bias, int64_t act, c10::optional<at::ScalarType> out_dtype,
                      int64_t force_path) {
  check_cuda(qa, "qa");
  c10::cuda::CUDAGuard g(qa.device());
  TORCH_CHECK(qa.scalar_type() == at::kChar && qbt.scalar_type() == at::kChar, "dlvk.gemm_i8: int8 operands");
  TORCH_CHECK(qa.dim() == 2 && qbt.dim() == 2 && qa.size(1) == qbt.size(1), "dlvk.gemm_i8: [M,K] x [N,K]");
  TORCH_CHECK(qa.stride(1) == 1 && qbt.stride(1) == 1, "dlvk.gemm_i8: K-contiguous operands");
  const int64_t M = qa.size(0), K = qa.size(1), N = qbt.size(0);
  auto C = at::empty({M, N}, qa.options().dtype(out_dtype.value_or(at::kFloat)));
  const float* bp = optf(bias);
  const bool tc = gemm_i8_tc_supported(qa.data_ptr(), qbt.data_ptr(), M, N, K, qa.stride(0), qbt.stride(0));
  const bool use_tc = force_path == 1 ? true : (force_path == 2 ? false : tc);
  if (use_tc) {
    TORCH_CHECK(tc, "dlvk.gemm_i8: tensor-core path not applicable");
    gemm_i8_tc(qa.data_ptr<int8_t>(), qbt.data_ptr<int8_t>(), sa.data_ptr<float>(), sb.data_ptr<float>(), bp,
               (int)act, C.data_ptr(), to_dtype(C), N, M, N, K, qa.stride(0), qbt.stride(0), stream(),
               device_error_word());
  } else {
    gemm_i8_simt(qa.data_ptr<int8_t>(), qbt.data_ptr<int8_t>(), sa.data_ptr<float>(), sb.data_ptr<float>(), bp,
                 (int)act, C.data_ptr(), to_dtype(C), N, M, N, K, qa.stride(0), qbt.stride(0), stream());
  }
  return C;
}

}  // namespace

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
        py::arg("dres") = py::none());
  m.def("dropout", &dropout_op, py::arg("x"), py::arg("p"), py::arg("stream_id") = 0, py::arg("seed") = 0,
        py::arg("step") = 0, py::arg("step_t") = py::none());
  m.def("embedding_fwd", &embedding_fwd_op);
  m.def("embedding_bwd", &embedding_bwd_op);
}

}  // namespace bind
}  // namespace dlvk
