// ATen-level wrappers of the dlvk kernels: argument checks, output
// allocation through PyTorch's caching allocator, launch on the current CUDA
// stream.  Shared by the Python module (csrc/bindings) and the C++ API
// (csrc/api), so both run exactly the same launch sequence for an op.
// Only ATen and CUDA headers: no Python.
#pragma once
#include <ATen/ATen.h>
#include <c10/util/Optional.h>
#include <cuda_runtime.h>

#include <utility>
#include <vector>

#include "dlvk/common.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace aten {

DType to_dtype(const at::Tensor& t);
void check_cuda(const at::Tensor& t, const char* name);
cudaStream_t stream();
at::Tensor unary_op(const at::Tensor& x, int64_t op, double a, double b, c10::optional<at::Tensor> out, c10::optional<at::ScalarType> out_dtype);
at::Tensor binary_op(const at::Tensor& x, const at::Tensor& y, int64_t op, c10::optional<at::Tensor> out);
at::Tensor bias_act_op(const at::Tensor& x, c10::optional<at::Tensor> bias, int64_t act);
at::Tensor reduce_op(const at::Tensor& x, int64_t op, double scale);
at::Tensor colsum_op(const at::Tensor& x, double scale, c10::optional<at::Tensor> out, bool accumulate, c10::optional<at::ScalarType> out_dtype);
at::Tensor rowsum_op(const at::Tensor& x, double scale);
at::Tensor transpose_op(const at::Tensor& x);
at::Tensor permute4_op(const at::Tensor& x, std::vector<int64_t> perm);
at::Tensor softmax_op(const at::Tensor& x, bool log_out);
at::Tensor softmax_bwd_op(const at::Tensor& y, const at::Tensor& dy);
std::vector<at::Tensor> softmax_ce_op(const at::Tensor& logits, const at::Tensor& target, double grad_scale, bool want_grad, bool in_place);
at::Tensor sum_scalar_op(const at::Tensor& v, double scale);
std::vector<at::Tensor> pointwise_loss_op(const at::Tensor& p, const at::Tensor& t, int64_t kind, double loss_scale, double grad_scale, bool want_grad);
GemmArgs fill_args(const at::Tensor& A, const at::Tensor& B, const at::Tensor& C);
int fp32_gemm_mode();
void set_fp32_gemm_mode(int mode);
bool gemm_tf32_ok(const at::Tensor& A, const at::Tensor& B);
void gemm_tf32_op(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const GemmArgs& args, bool three_pass,
                  int max_ctas);
at::Tensor gemm_op(const at::Tensor& A, const at::Tensor& B, c10::optional<at::Tensor> bias, int64_t act, double alpha, double beta, c10::optional<at::Tensor> out, c10::optional<at::ScalarType> out_dtype, int64_t force_path, int64_t max_ctas, c10::optional<at::Tensor> residual, c10::optional<at::Tensor> relu_mask, c10::optional<at::Tensor> colsum_out, double colsum_scale, bool colsum_accumulate, c10::optional<at::Tensor> relu_bits_out = c10::nullopt, c10::optional<at::Tensor> relu_bits = c10::nullopt);
bool gemm_tc_ok(const at::Tensor& A, const at::Tensor& B);
void optim_advance_op(const at::Tensor& hyper);
void optim_update_op(int64_t kind, const at::Tensor& hyper, const at::Tensor& p, const at::Tensor& grad, c10::optional<at::Tensor> m, c10::optional<at::Tensor> v, c10::optional<at::Tensor> p_bf16, double extra_scale, int64_t max_ctas);
void grad_stats_op(const at::Tensor& g, double scale, double max_norm, const at::Tensor& sumsq, c10::optional<at::Tensor> flag, c10::optional<at::Tensor> clip, bool accumulate, const at::Tensor& scratch, c10::optional<at::Tensor> scale_dev);
void scaler_update_op(const at::Tensor& scale, const at::Tensor& good_steps, const at::Tensor& found_inf, double growth, double backoff, int64_t interval, double smin, double smax, c10::optional<at::Tensor> inv_scale);
int64_t optim_hyper_bytes();
const float* optf(const c10::optional<at::Tensor>& t);
float* optfm(const c10::optional<at::Tensor>& t);
ConvDesc conv_desc(const at::Tensor& x, const at::Tensor& w, int64_t stride, int64_t pad);
DropoutDesc drop_desc(double p, int64_t stream_id, int64_t seed, int64_t step, const c10::optional<at::Tensor>& step_t);
at::Tensor to_nhwc(const at::Tensor& x);
at::Tensor pack_conv_weights(const at::Tensor& w, const ConvDesc& d, bool dgrad);
const __nv_bfloat16* bf(const at::Tensor& t);
at::Tensor conv2d_fwd_op(const at::Tensor& x, const at::Tensor& w, c10::optional<at::Tensor> bias, int64_t stride, int64_t pad, bool relu);
at::Tensor conv2d_dgrad_op(const at::Tensor& gy, const at::Tensor& w, std::vector<int64_t> xshape, int64_t stride, int64_t pad, c10::optional<at::Tensor> relu_src);
void conv2d_wgrad_op(const at::Tensor& x, const at::Tensor& gy, const at::Tensor& dw, c10::optional<at::Tensor> db, int64_t stride, int64_t pad, bool accumulate);
std::vector<at::Tensor> maxpool_fwd_op(const at::Tensor& x, int64_t k, int64_t stride);
at::Tensor maxpool_bwd_op(const at::Tensor& gy, const at::Tensor& idx, int64_t H, int64_t W, int64_t k, int64_t stride);
at::Tensor avgpool_fwd_op(const at::Tensor& x, int64_t k, int64_t stride, int64_t pad);
at::Tensor avgpool_bwd_op(const at::Tensor& gy, int64_t H, int64_t W, int64_t k, int64_t stride, int64_t pad);
std::vector<at::Tensor> batchnorm_fwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> beta, c10::optional<at::Tensor> run_mean, c10::optional<at::Tensor> run_var, double momentum, double eps, bool training, bool relu, double p, int64_t stream_id, int64_t seed, int64_t step, c10::optional<at::Tensor> step_t);
at::Tensor batchnorm_bwd_op(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& mean, const at::Tensor& rstd, c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> beta, c10::optional<at::Tensor> dgamma, c10::optional<at::Tensor> dbeta, bool accumulate, bool relu, double p, int64_t stream_id, int64_t seed, int64_t step, c10::optional<at::Tensor> step_t);
std::vector<at::Tensor> layernorm_fwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> beta, double eps);
at::Tensor layernorm_bwd_op(const at::Tensor& x, c10::optional<at::Tensor> gamma, const at::Tensor& mean, const at::Tensor& rstd, const at::Tensor& dy, c10::optional<at::Tensor> dgamma, c10::optional<at::Tensor> dbeta, bool accumulate, c10::optional<at::Tensor> dres, c10::optional<at::Tensor> dres_colsum = c10::nullopt, bool dres_colsum_accumulate = false);
at::Tensor dropout_op(const at::Tensor& x, double p, int64_t stream_id, int64_t seed, int64_t step, c10::optional<at::Tensor> step_t);
at::Tensor embedding_fwd_op(const at::Tensor& ids, const at::Tensor& table);
void embedding_bwd_op(const at::Tensor& ids, const at::Tensor& dy, const at::Tensor& dtable);
std::vector<at::Tensor> quantize_rows_op(const at::Tensor& x);
at::Tensor gemm_i8_op(const at::Tensor& qa, const at::Tensor& qbt, const at::Tensor& sa, const at::Tensor& sb, c10::optional<at::Tensor> bias, int64_t act, c10::optional<at::ScalarType> out_dtype, int64_t force_path);

}  // namespace aten
}  // namespace dlvk
