// ATen-level wrappers of the layer kernels: convolution, pooling, batch /
// layer norm, dropout, embedding and the int8 quantised GEMM (declared in
// dlvk/aten_ops.h).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "dlvk/aten_ops.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace aten {

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

// 1x1 filter, stride 1, no padding: in NCHW the convolution is a batched
// GEMM over the tensors as they are (no NHWC copy, no im2col gather):
//   forward  y[n] (Cout x HW) = W (Cout x Cin) . x[n] (Cin x HW), bias per row
//   dgrad    dx[n] (Cin x HW) = W^T (Cin x Cout) . dy[n] (Cout x HW)
//   wgrad    dW (Cout x Cin) = sum_n dy[n] (Cout x HW) . x[n]^T (HW x Cin)
// with W shared by every image (zero batch stride).  Needs bf16 and rows
// whose byte strides are multiples of 16 (channels and H*W multiples of 8).
bool conv1x1_gemm_ok(const ConvDesc& d) {
  const int64_t hw = (int64_t)d.H * d.W;
  return d.KH == 1 && d.KW == 1 && d.stride == 1 && d.pad == 0 && d.Cin % 8 == 0 && d.Cout % 8 == 0 &&
         hw % 8 == 0 && hw >= 16 && conv2d_tc_supported(DType::BF16, d);
}

void run_gemm_tc(DType out_dt, const GemmArgs& a, const at::Tensor& like) {
  TORCH_CHECK(gemm_tc_supported(a), "dlvk.conv2d: 1x1 GEMM operands not tensor-core aligned");
  const int64_t wsf = gemm_tc_workspace_floats(a, 0, out_dt);
  at::Tensor ws = wsf > 0 ? at::empty({wsf}, like.options().dtype(at::kFloat)) : at::Tensor();
  gemm_tc(out_dt, a, stream(), device_error_word(), 0, wsf > 0 ? ws.data_ptr<float>() : nullptr, wsf);
}

at::Tensor conv2d_fwd_op(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias, int64_t stride,
                         int64_t pad, bool relu) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), wc = w.contiguous().to(x.scalar_type());
  auto d = conv_desc(xc, wc, stride, pad);
  auto y = at::empty({d.N, d.Cout, d.Ho, d.Wo}, xc.options());
  if (xc.scalar_type() == at::kBFloat16 && conv1x1_gemm_ok(d)) {
    const int64_t hw = (int64_t)d.H * d.W;
    GemmArgs a;
    a.A = wc.data_ptr();
    a.B = xc.data_ptr();
    a.C = y.data_ptr();
    a.M = d.Cout;
    a.N = hw;
    a.K = d.Cin;
    a.sam = d.Cin;
    a.sak = 1;
    a.sbk = hw;
    a.sbn = 1;
    a.ldc = hw;
    a.batch = d.N;
    a.batch_stride_a = 0;
    a.batch_stride_b = (int64_t)d.Cin * hw;
    a.batch_stride_c = (int64_t)d.Cout * hw;
    a.row_bias = optf(bias);
    a.act = relu ? ACT_RELU : ACT_NONE;
    run_gemm_tc(DType::BF16, a, xc);
    return y;
  }
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
  if (gc.scalar_type() == at::kBFloat16 && conv1x1_gemm_ok(d)) {
    const int64_t hw = (int64_t)d.H * d.W;
    GemmArgs a;
    a.A = wc.data_ptr();  // W^T: [Cin x Cout] read M-major from W [Cout x Cin]
    a.B = gc.data_ptr();
    a.C = dx.data_ptr();
    a.M = d.Cin;
    a.N = hw;
    a.K = d.Cout;
    a.sam = 1;
    a.sak = d.Cin;
    a.sbk = hw;
    a.sbn = 1;
    a.ldc = hw;
    a.batch = d.N;
    a.batch_stride_a = 0;
    a.batch_stride_b = (int64_t)d.Cout * hw;
    a.batch_stride_c = (int64_t)d.Cin * hw;
    if (rs) {
      a.relu_mask = rs;
      a.ldm = hw;
      a.batch_stride_m = (int64_t)d.Cin * hw;
    }
    run_gemm_tc(DType::BF16, a, gc);
    return dx;
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
  if (xc.scalar_type() == at::kBFloat16 && conv1x1_gemm_ok(d)) {
    TORCH_CHECK(gc.size(2) == d.Ho && gc.size(3) == d.Wo, "dlvk.conv2d_wgrad: grad shape");
    const int64_t hw = (int64_t)d.H * d.W;
    // Per-image products [N, Cout, Cin] in fp32, then summed over the images
    // in image order (deterministic) into dW.
    auto part = at::empty({d.N, d.Cout, d.Cin}, xc.options().dtype(at::kFloat));
    GemmArgs a;
    a.A = gc.data_ptr();
    a.B = xc.data_ptr();  // x[n]^T: [HW x Cin] read K-major from x[n] [Cin x HW]
    a.C = part.data_ptr();
    a.M = d.Cout;
    a.N = d.Cin;
    a.K = hw;
    a.sam = hw;
    a.sak = 1;
    a.sbk = 1;
    a.sbn = hw;
    a.ldc = d.Cin;
    a.batch = d.N;
    a.batch_stride_a = (int64_t)d.Cout * hw;
    a.batch_stride_b = (int64_t)d.Cin * hw;
    a.batch_stride_c = (int64_t)d.Cout * d.Cin;
    run_gemm_tc(DType::F32, a, xc);
    const int64_t cols = (int64_t)d.Cout * d.Cin;
    const int64_t ns = colsum_scratch_floats(d.N, cols);
    at::Tensor scr = ns > 0 ? at::empty({ns}, part.options()) : at::Tensor();
    colsum(DType::F32, DType::F32, part.data_ptr(), d.N, cols, 1.f, dw.data_ptr<float>(), accumulate,
           ns > 0 ? scr.data_ptr<float>() : nullptr, stream());
    if (db.has_value()) {
      // db[c] = sum over images and pixels of dy[n, c, :]: row sums, then a column sum over images.
      auto rows = at::empty({(int64_t)d.N * d.Cout}, part.options());
      rowsum(DType::BF16, gc.data_ptr(), (int64_t)d.N * d.Cout, hw, 1.f, rows.data_ptr<float>(), stream());
      const int64_t ns2 = colsum_scratch_floats(d.N, d.Cout);
      at::Tensor scr2 = ns2 > 0 ? at::empty({ns2}, part.options()) : at::Tensor();
      colsum(DType::F32, DType::F32, rows.data_ptr(), d.N, d.Cout, 1.f, db->data_ptr<float>(), accumulate,
             ns2 > 0 ? scr2.data_ptr<float>() : nullptr, stream());
    }
    return;
  }
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
                            c10::optional<at::Tensor> dbeta, bool accumulate, c10::optional<at::Tensor> dres,
                            c10::optional<at::Tensor> dres_colsum, bool dres_colsum_accumulate) {
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
  TORCH_CHECK(!dres_colsum.has_value() || (dres.has_value() && dres_colsum->numel() == D),
              "dlvk.layernorm_bwd: dres_colsum needs dres and D elements");
  layernorm_bwd(to_dtype(xc), xc.data_ptr(), optf(gamma), mean.data_ptr<float>(), rstd.data_ptr<float>(),
                dyc.data_ptr(), dx.data_ptr(), optfm(dgamma), optfm(dbeta), accumulate, R, (int)D,
                scratch.data_ptr<float>(), stream(), dres.has_value() ? drc.data_ptr() : nullptr,
                optfm(dres_colsum), dres_colsum_accumulate);
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

}  // namespace aten
}  // namespace dlvk
