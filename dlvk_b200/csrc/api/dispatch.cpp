// Op dispatch of the C++ API: CUDA tensors -> sm_100a kernels (ATen op
// layer), CPU tensors -> ATen reference path.  Each CPU branch restates the
// Python package's CPU path of the same op (dlvk_b200/ops/core.py,
// dlvk_b200/ops/nn.py, dlvk_b200/optim.py) with the same ATen calls in the
// same order, so the two front ends produce the same bits.
#include "dispatch.h"

#include <cmath>

#include "dlvk/aten_ops.h"
#include "dlvk/oracle.h"

namespace dlvk {
namespace api {

namespace {
at::Tensor zeros_like_f(const at::Tensor& t) { return at::zeros_like(t); }

at::Tensor unary_ref(const at::Tensor& x, int op, double a, double b) {
  at::Tensor xf = x.to(at::kFloat);
  switch (op) {
    case UN_RELU: return at::relu(xf);
    case UN_SIGMOID: return at::sigmoid(xf);
    case UN_TANH: return at::tanh(xf);
    case UN_SCALE: return xf * a;
    case UN_CLAMP: return xf.clamp(a, b);
    case UN_SQRT: return xf.sqrt();
    case UN_COPY: return xf;
    case UN_SQUARE: return xf * xf;
    case UN_ADD_SCALAR: return xf + a;
    case UN_ABS: return xf.abs();
    case UN_EXP: return xf.exp();
    case UN_LOG: return xf.log();
    case UN_GELU: return at::gelu(xf);
    default: TORCH_CHECK(false, "dlvk: unknown unary op ", op);
  }
}

at::Tensor binary_ref(const at::Tensor& x, const at::Tensor& y, int op) {
  at::Tensor xf = x.to(at::kFloat), yf = y.to(at::kFloat);
  switch (op) {
    case BIN_ADD: return xf + yf;
    case BIN_SUB: return xf - yf;
    case BIN_MUL: return xf * yf;
    case BIN_DIV: {
      // the reference's guarded divide (shaders/tensor_divide.comp:29-34)
      at::Tensor guard = yf.abs() < 1e-8;
      at::Tensor sign = at::where(xf >= 0, at::ones_like(xf), -at::ones_like(xf));
      return at::where(guard, sign * 1e8, xf / at::where(guard, at::ones_like(yf), yf));
    }
    case BIN_MAX: return at::maximum(xf, yf);
    case BIN_MIN: return at::minimum(xf, yf);
    case BIN_RELU_BWD: return at::where(yf > 0, xf, zeros_like_f(xf));
    case BIN_SIGMOID_BWD: return xf * yf * (1 - yf);
    case BIN_TANH_BWD: return xf * (1 - yf * yf);
    default: TORCH_CHECK(false, "dlvk: unknown binary op ", op);
  }
}
}  // namespace

at::Tensor unary(const at::Tensor& x, int op, double a, double b) {
  if (x.is_cuda()) return aten::unary_op(x, op, a, b, c10::nullopt, c10::nullopt);
  return unary_ref(x, op, a, b).to(x.scalar_type());
}

at::Tensor binary(const at::Tensor& x, const at::Tensor& y, int op) {
  if (x.is_cuda()) return aten::binary_op(x, y.scalar_type() == x.scalar_type() ? y : y.to(x.scalar_type()), op,
                                          c10::nullopt);
  return binary_ref(x, y, op).to(x.scalar_type());
}

at::Tensor bias_act(const at::Tensor& x, const at::Tensor& bias) {
  if (x.is_cuda()) return aten::bias_act_op(x, bias, UN_COPY);
  return (x.to(at::kFloat) + bias.to(at::kFloat)).to(x.scalar_type());
}

at::Tensor reduce(const at::Tensor& x, int op, double scale) {
  if (x.is_cuda()) return aten::reduce_op(x, op, scale);
  at::Tensor xf = x.to(at::kFloat);
  switch (op) {
    case RED_SUM: return xf.sum() * scale;
    case RED_MAX: return xf.max() * scale;
    case RED_MIN: return xf.min() * scale;
    case RED_SUMSQ: return (xf * xf).sum() * scale;
    case RED_ABSMAX: return xf.abs().max() * scale;
    default: TORCH_CHECK(false, "dlvk: unknown reduction ", op);
  }
}

at::Tensor colsum(const at::Tensor& x, double scale, OptT out, bool accumulate) {
  if (x.is_cuda()) return aten::colsum_op(x, scale, out, accumulate, c10::nullopt);
  const int64_t cols = x.size(-1);
  at::Tensor s = x.reshape({-1, cols}).to(at::kFloat).sum(0) * scale;
  if (out.has_value()) {
    if (accumulate) out->add_(s.to(out->scalar_type()));
    else out->copy_(s);
    return *out;
  }
  return s;
}

at::Tensor transpose(const at::Tensor& x) {
  if (x.is_cuda()) return aten::transpose_op(x);
  return x.transpose(-1, -2).contiguous();
}

at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, OptT bias, int act, double alpha, double beta, OptT out,
                OptT relu_mask) {
  if (a.is_cuda())
    return aten::gemm_op(a, b, bias, act, alpha, beta, out, c10::nullopt, 0, 0, c10::nullopt, relu_mask,
                         c10::nullopt, 1.0, false);
  at::Tensor c = at::matmul(a.to(at::kFloat), b.to(at::kFloat)) * alpha;
  if (beta != 0.0 && out.has_value()) c = c + out->to(at::kFloat) * beta;
  if (bias.has_value()) c = c + bias->to(at::kFloat);
  if (act == ACT_RELU) c = at::relu(c);
  else if (act == ACT_GELU) c = at::gelu(c);
  if (relu_mask.has_value()) c = at::where(relu_mask->to(at::kFloat) > 0, c, at::zeros_like(c));
  if (out.has_value()) {
    out->copy_(c);
    return *out;
  }
  return c.to(a.scalar_type());
}

at::Tensor softmax(const at::Tensor& x) {
  if (x.is_cuda()) return aten::softmax_op(x, false);
  return at::softmax(x.to(at::kFloat), -1).to(x.scalar_type());
}

at::Tensor softmax_bwd(const at::Tensor& y, const at::Tensor& dy) {
  if (y.is_cuda()) return aten::softmax_bwd_op(y, dy);
  at::Tensor yf = y.to(at::kFloat), dyf = dy.to(at::kFloat);
  return (yf * (dyf - (yf * dyf).sum(-1, true))).to(y.scalar_type());
}

std::pair<at::Tensor, at::Tensor> softmax_ce(const at::Tensor& logits, const at::Tensor& target, double grad_scale) {
  if (logits.is_cuda()) {
    at::Tensor tg = target;
    if (!tg.is_floating_point() && tg.scalar_type() != at::kInt) tg = tg.to(at::kInt);
    auto r = aten::softmax_ce_op(logits.contiguous(), tg, grad_scale, true, false);
    return {r[0], r[1]};
  }
  const int64_t cols = logits.size(-1);
  at::Tensor x = logits.reshape({-1, cols}).to(at::kFloat);
  at::Tensor lse = at::logsumexp(x, -1);
  at::Tensor p = at::softmax(x, -1);
  at::Tensor loss, g;
  if (!target.is_floating_point()) {
    at::Tensor lab = target.reshape({-1}).to(at::kLong);
    at::Tensor valid = lab >= 0;
    at::Tensor t = at::zeros_like(x);
    t.index_put_({valid, lab.index({valid})}, 1.0);
    loss = at::where(valid, lse - x.gather(1, lab.clamp_min(0).unsqueeze(1)).select(1, 0), at::zeros_like(lse));
    g = (p - t) * grad_scale;
    g.index_put_({valid.logical_not()}, 0);
  } else {
    at::Tensor t = target.reshape({-1, cols}).to(at::kFloat);
    loss = (t * (lse.unsqueeze(1) - x)).sum(-1);
    g = (p - t) * grad_scale;
  }
  return {loss, g.to(logits.scalar_type()).reshape(logits.sizes())};
}

at::Tensor sum_scalar(const at::Tensor& v, double scale) {
  if (v.is_cuda()) return aten::sum_scalar_op(v, scale);
  return v.to(at::kFloat).sum() * scale;
}

std::pair<at::Tensor, at::Tensor> pointwise_loss(const at::Tensor& p, const at::Tensor& t, int kind,
                                                 double loss_scale, double grad_scale, bool want_grad) {
  if (p.is_cuda()) {
    auto r = aten::pointwise_loss_op(p, t, kind, loss_scale, grad_scale, want_grad);
    return {r[0], r[1]};
  }
  at::Tensor pf = p.to(at::kFloat), tf = t.to(at::kFloat);
  at::Tensor loss, g;
  if (kind == LOSS_MSE) {
    at::Tensor d = pf - tf;
    loss = (d * d).sum() * loss_scale;
    g = d * 2 * grad_scale;
  } else {
    at::Tensor pc = pf.clamp(1e-7, 1 - 1e-7);
    loss = (-(tf * pc.log() + (1 - tf) * (1 - pc).log())).sum() * loss_scale;
    g = (pc - tf) / (pc * (1 - pc)) * grad_scale;
  }
  return {loss, want_grad ? g.to(p.scalar_type()) : at::Tensor()};
}

// ---------------------------------------------------------------- layers
at::Tensor conv2d_fwd(const at::Tensor& x, const at::Tensor& w, OptT bias, int stride, int pad, bool relu) {
  if (x.is_cuda()) return aten::conv2d_fwd_op(x, w, bias, stride, pad, relu);
  at::Tensor y = at::conv2d(x.to(at::kFloat), w.to(at::kFloat),
                            bias.has_value() ? c10::optional<at::Tensor>(bias->to(at::kFloat)) : c10::nullopt,
                            {stride, stride}, {pad, pad});
  if (relu) y = at::relu(y);
  return y.to(x.scalar_type());
}

at::Tensor conv2d_dgrad(const at::Tensor& gy, const at::Tensor& w, const std::vector<int64_t>& xshape, int stride,
                        int pad, OptT relu_src) {
  if (gy.is_cuda()) return aten::conv2d_dgrad_op(gy, w, xshape, stride, pad, relu_src);
  // d/dx of conv2d: the transposed convolution of gy with w (output padding
  // recovers the input extent for strided layers).
  const int64_t hout = (xshape[2] + 2 * pad - w.size(2)) / stride + 1;
  const int64_t wout = (xshape[3] + 2 * pad - w.size(3)) / stride + 1;
  const int64_t oph = xshape[2] - ((hout - 1) * stride - 2 * pad + w.size(2));
  const int64_t opw = xshape[3] - ((wout - 1) * stride - 2 * pad + w.size(3));
  at::Tensor dx = at::conv_transpose2d(gy.to(at::kFloat), w.to(at::kFloat), c10::nullopt, {stride, stride},
                                       {pad, pad}, {oph, opw});
  if (relu_src.has_value()) dx = at::where(relu_src->to(at::kFloat) > 0, dx, at::zeros_like(dx));
  return dx.to(gy.scalar_type());
}

void conv2d_wgrad(const at::Tensor& x, const at::Tensor& gy, at::Tensor& dw, OptT db, int stride, int pad,
                  bool accumulate) {
  if (x.is_cuda()) {
    aten::conv2d_wgrad_op(x, gy, dw, db, stride, pad, accumulate);
    return;
  }
  // dW[o, c, kh, kw] = sum over n, y of gy[n, o, y] * x[n, c, y*s + k - p]:
  // the convolution of x (channels as batch) with gy (images as channels).
  at::Tensor xt = x.to(at::kFloat).transpose(0, 1);
  at::Tensor gt = gy.to(at::kFloat).transpose(0, 1);
  at::Tensor gw = at::conv2d(xt, gt, c10::nullopt, {1, 1}, {pad, pad}, {stride, stride}).transpose(0, 1);
  gw = gw.narrow(2, 0, dw.size(2)).narrow(3, 0, dw.size(3));
  at::Tensor gb = gy.to(at::kFloat).sum({0, 2, 3});
  if (accumulate) {
    dw.add_(gw);
    if (db.has_value()) db->add_(gb);
  } else {
    dw.copy_(gw);
    if (db.has_value()) db->copy_(gb);
  }
}

std::pair<at::Tensor, at::Tensor> maxpool_fwd(const at::Tensor& x, int k, int stride) {
  if (x.is_cuda()) {
    auto r = aten::maxpool_fwd_op(x, k, stride);
    return {r[0], r[1]};
  }
  auto r = at::max_pool2d_with_indices(x.to(at::kFloat), {k, k}, {stride, stride});
  return {std::get<0>(r).to(x.scalar_type()), std::get<1>(r).to(at::kInt)};
}

at::Tensor maxpool_bwd(const at::Tensor& gy, const at::Tensor& idx, int H, int W, int k, int stride) {
  if (gy.is_cuda()) return aten::maxpool_bwd_op(gy, idx, H, W, k, stride);
  const int64_t n = gy.size(0), c = gy.size(1);
  at::Tensor dx = at::zeros({n, c, (int64_t)H * W}, gy.options().dtype(at::kFloat));
  dx.scatter_add_(2, idx.reshape({n, c, -1}).to(at::kLong), gy.to(at::kFloat).reshape({n, c, -1}));
  return dx.reshape({n, c, H, W}).to(gy.scalar_type());
}

at::Tensor avgpool_fwd(const at::Tensor& x, int k, int stride) {
  if (x.is_cuda()) return aten::avgpool_fwd_op(x, k, stride, 0);
  return at::avg_pool2d(x.to(at::kFloat), {k, k}, {stride, stride}, {0, 0}, false, false).to(x.scalar_type());
}

at::Tensor avgpool_bwd(const at::Tensor& gy, int H, int W, int k, int stride) {
  if (gy.is_cuda()) return aten::avgpool_bwd_op(gy, H, W, k, stride, 0);
  at::Tensor x = at::zeros({gy.size(0), gy.size(1), H, W}, gy.options().dtype(at::kFloat));
  return at::avg_pool2d_backward(gy.to(at::kFloat), x, {k, k}, {stride, stride}, {0, 0}, false, false, c10::nullopt)
      .to(gy.scalar_type());
}

std::vector<at::Tensor> batchnorm_fwd(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta,
                                      at::Tensor& run_mean, at::Tensor& run_var, double momentum, double eps,
                                      bool training) {
  if (x.is_cuda())
    return aten::batchnorm_fwd_op(x, gamma, beta, run_mean, run_var, momentum, eps, training, false, 0.0, 0, 0, 0,
                                  c10::nullopt);
  const int64_t C = x.size(1);
  at::Tensor xf = x.to(at::kFloat);
  std::vector<int64_t> dims{0}, shape{1, C};
  for (int64_t d = 2; d < x.dim(); ++d) {
    dims.push_back(d);
    shape.push_back(1);
  }
  at::Tensor mean, var;
  if (training) {
    mean = xf.mean(dims);
    var = xf.var(dims, false);
    run_mean.mul_(1 - momentum).add_(mean * momentum);
    run_var.mul_(1 - momentum).add_(var * momentum);
  } else {
    mean = run_mean.to(at::kFloat);
    var = run_var.to(at::kFloat);
  }
  at::Tensor rstd = at::rsqrt(var + eps);
  at::Tensor y = (xf - mean.reshape(shape)) * rstd.reshape(shape);
  y = y * gamma.reshape(shape) + beta.reshape(shape);
  return {y.to(x.scalar_type()), mean, rstd};
}

at::Tensor batchnorm_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& mean, const at::Tensor& rstd,
                         const at::Tensor& gamma, const at::Tensor& beta, at::Tensor& dgamma, at::Tensor& dbeta,
                         bool accumulate) {
  if (x.is_cuda())
    return aten::batchnorm_bwd_op(x, dy, mean, rstd, gamma, beta, dgamma, dbeta, accumulate, false, 0.0, 0, 0, 0,
                                  c10::nullopt);
  const int64_t C = x.size(1);
  std::vector<int64_t> dims{0}, shape{1, C};
  for (int64_t d = 2; d < x.dim(); ++d) {
    dims.push_back(d);
    shape.push_back(1);
  }
  at::Tensor xh = (x.to(at::kFloat) - mean.reshape(shape)) * rstd.reshape(shape);
  at::Tensor g = dy.to(at::kFloat);
  at::Tensor gm = gamma.reshape(shape);
  at::Tensor sg = g.sum(dims);
  at::Tensor sgx = (g * xh).sum(dims);
  const double cnt = (double)(x.numel() / C);
  at::Tensor dx = gm * rstd.reshape(shape) * (g - sg.reshape(shape) / cnt - xh * sgx.reshape(shape) / cnt);
  if (accumulate) {
    dgamma.add_(sgx);
    dbeta.add_(sg);
  } else {
    dgamma.copy_(sgx);
    dbeta.copy_(sg);
  }
  return dx.to(x.scalar_type());
}

at::Tensor dropout(const at::Tensor& x, double p, int64_t site, uint64_t seed, int64_t step) {
  if (x.is_cuda()) return aten::dropout_op(x, p, site, (int64_t)seed, step, c10::nullopt);
  at::Tensor keep = at::empty({x.numel()}, x.options().dtype(at::kByte));
  ref::dropout_mask(keep.data_ptr<uint8_t>(), x.numel(), (float)p, seed, (uint32_t)site, (uint32_t)step);
  keep = keep.to(at::kBool).reshape(x.sizes());
  return at::where(keep, x.to(at::kFloat) / (1 - p), at::zeros_like(x, x.options().dtype(at::kFloat)))
      .to(x.scalar_type());
}

// ---------------------------------------------------------------- optimizers
void optim_update(int kind, const at::Tensor& hyper_dev, const CpuHyper& h, at::Tensor& p, const at::Tensor& g_in,
                  OptT m, OptT v) {
  if (p.is_cuda()) {
    aten::optim_update_op(kind, hyper_dev, p, g_in, m, v, c10::nullopt, 1.0, 0);
    return;
  }
  // Gradient times the (unit) loss-scale and clip factors, as the Python CPU path does.
  at::Tensor g = g_in.to(at::kFloat) * 1.0 * 1.0;
  const double lr = h.lr;
  if (h.weight_decay != 0.0) g = g + p * h.weight_decay;
  const int64_t t = h.step;
  if (kind == OPT_ADAM) {
    m->mul_(h.beta1).add_(g * (1 - h.beta1));
    v->mul_(h.beta2).add_(g * (1 - h.beta2) * g);
    const double bc1 = h.bias_correction ? 1.0 / (1 - std::pow(h.beta1, (double)t)) : 1.0;
    const double bc2 = h.bias_correction ? 1.0 / (1 - std::pow(h.beta2, (double)t)) : 1.0;
    p.sub_((*m * bc1) * lr / (at::sqrt(*v * bc2) + h.eps));
  } else if (kind == OPT_SGD) {
    if (h.momentum != 0.0) {
      m->mul_(h.momentum).add_(g);
      p.sub_(*m * lr);
    } else {
      p.sub_(g * lr);
    }
  } else {
    v->mul_(h.alpha).add_(g * (1 - h.alpha) * g);
    p.sub_(g * lr / (at::sqrt(*v) + h.eps));
  }
}

}  // namespace api
}  // namespace dlvk
