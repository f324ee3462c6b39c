// Op dispatch of the C++ API (private header).  A CUDA tensor goes to the
// sm_100a kernels through the ATen op layer (dlvk/aten_ops.h), the same
// launches the Python package makes; a CPU tensor takes a plain ATen
// reference path that restates, op for op, the Python package's CPU path
// (dlvk_b200/ops/core.py, dlvk_b200/ops/nn.py), so the two front ends agree
// bit for bit on either device.
#pragma once
#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include <utility>

#include "dlvk/kernels.h"

namespace dlvk {
namespace api {

using OptT = c10::optional<at::Tensor>;

at::Tensor unary(const at::Tensor& x, int op, double a = 0.0, double b = 0.0);
at::Tensor binary(const at::Tensor& x, const at::Tensor& y, int op);
at::Tensor bias_act(const at::Tensor& x, const at::Tensor& bias);
at::Tensor reduce(const at::Tensor& x, int op, double scale = 1.0);
// out (+)= scale * column sums of x viewed as [rows, cols]; returns out or a new [cols] fp32 tensor.
at::Tensor colsum(const at::Tensor& x, double scale = 1.0, OptT out = c10::nullopt, bool accumulate = false);
at::Tensor transpose(const at::Tensor& x);
// act(alpha * a @ b + beta * out + bias), zeroed where relu_mask <= 0.
at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, OptT bias = c10::nullopt, int act = ACT_NONE,
                double alpha = 1.0, double beta = 0.0, OptT out = c10::nullopt, OptT relu_mask = c10::nullopt);
at::Tensor softmax(const at::Tensor& x);
at::Tensor softmax_bwd(const at::Tensor& y, const at::Tensor& dy);
// Fused softmax + cross-entropy from logits: (per-row loss fp32, dlogits).
// target: int32 class ids [rows] or fp32 probabilities [rows, cols].
std::pair<at::Tensor, at::Tensor> softmax_ce(const at::Tensor& logits, const at::Tensor& target, double grad_scale);
at::Tensor sum_scalar(const at::Tensor& v, double scale);
std::pair<at::Tensor, at::Tensor> pointwise_loss(const at::Tensor& p, const at::Tensor& t, int kind,
                                                 double loss_scale, double grad_scale, bool want_grad);

at::Tensor conv2d_fwd(const at::Tensor& x, const at::Tensor& w, OptT bias, int stride, int pad, bool relu);
at::Tensor conv2d_dgrad(const at::Tensor& gy, const at::Tensor& w, const std::vector<int64_t>& xshape, int stride,
                        int pad, OptT relu_src);
void conv2d_wgrad(const at::Tensor& x, const at::Tensor& gy, at::Tensor& dw, OptT db, int stride, int pad,
                  bool accumulate);
std::pair<at::Tensor, at::Tensor> maxpool_fwd(const at::Tensor& x, int k, int stride);
at::Tensor maxpool_bwd(const at::Tensor& gy, const at::Tensor& idx, int H, int W, int k, int stride);
at::Tensor avgpool_fwd(const at::Tensor& x, int k, int stride);
at::Tensor avgpool_bwd(const at::Tensor& gy, int H, int W, int k, int stride);
// Returns (y, batch mean, batch rstd).
std::vector<at::Tensor> batchnorm_fwd(const at::Tensor& x, const at::Tensor& gamma, const at::Tensor& beta,
                                      at::Tensor& run_mean, at::Tensor& run_var, double momentum, double eps,
                                      bool training);
at::Tensor batchnorm_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& mean, const at::Tensor& rstd,
                         const at::Tensor& gamma, const at::Tensor& beta, at::Tensor& dgamma, at::Tensor& dbeta,
                         bool accumulate);
// Inverted dropout with the framework's Philox stream (seed, site, step).
at::Tensor dropout(const at::Tensor& x, double p, int64_t site, uint64_t seed, int64_t step);

// Optimizer update over flat fp32 buffers (p, grad, m, v): on CUDA the
// optim.cu kernel reading the device hyper block; on CPU the reference
// formulas of the Python package's CPU optimizer.
struct CpuHyper {
  double lr, beta1, beta2, eps, weight_decay, momentum, alpha;
  bool bias_correction;
  int64_t step;
};
void optim_update(int kind, const at::Tensor& hyper_dev, const CpuHyper& h, at::Tensor& p, const at::Tensor& g,
                  OptT m, OptT v);

}  // namespace api
}  // namespace dlvk
