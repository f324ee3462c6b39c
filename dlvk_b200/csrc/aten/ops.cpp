// ATen-level wrappers of the elementwise, reduction, softmax / loss, GEMM
// and optimizer kernels (declared in dlvk/aten_ops.h).  Every op launches on
// the current CUDA stream of its tensors' device, takes strided views where
// the kernel supports them, and allocates outputs through PyTorch's caching
// allocator (so the ops are CUDA-graph capturable).
#include <ATen/ATen.h>
#include <cstdlib>
#include <string>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "dlvk/aten_ops.h"
#include "dlvk/kernels.h"

namespace dlvk {
namespace aten {

DType to_dtype(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return DType::F32;
    case at::kBFloat16: return DType::BF16;
    case at::kHalf: return DType::F16;
    case at::kInt: return DType::I32;
    case at::kChar: return DType::I8;
    case at::kByte: return DType::U8;
    case at::kLong: return DType::I64;
    default: TORCH_CHECK(false, "dlvk: unsupported dtype ", t.scalar_type());
  }
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "dlvk: ", name, " must be a CUDA tensor (the native kernels run on the GPU only)");
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// ---- elementwise ----
at::Tensor unary_op(const at::Tensor& x, int64_t op, double a, double b, c10::optional<at::Tensor> out,
                    c10::optional<at::ScalarType> out_dtype) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  at::Tensor y = out.has_value() ? *out : at::empty_like(xc, xc.options().dtype(out_dtype.value_or(xc.scalar_type())));
  TORCH_CHECK(y.is_contiguous() && y.numel() == xc.numel(), "dlvk.unary: bad out");
  unary(to_dtype(xc), to_dtype(y), xc.data_ptr(), y.data_ptr(), xc.numel(), (int)op, (float)a, (float)b, stream());
  return y;
}

at::Tensor binary_op(const at::Tensor& x, const at::Tensor& y, int64_t op, c10::optional<at::Tensor> out) {
  check_cuda(x, "x");
  check_cuda(y, "y");
  TORCH_CHECK(x.sizes() == y.sizes(), "dlvk.binary: shape mismatch ", x.sizes(), " vs ", y.sizes());
  TORCH_CHECK(x.scalar_type() == y.scalar_type(), "dlvk.binary: dtype mismatch");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous(), yc = y.contiguous();
  at::Tensor z = out.has_value() ? *out : at::empty_like(xc);
  TORCH_CHECK(z.is_contiguous() && z.numel() == xc.numel(), "dlvk.binary: bad out");
  binary(to_dtype(xc), xc.data_ptr(), yc.data_ptr(), z.data_ptr(), xc.numel(), (int)op, stream());
  return z;
}

at::Tensor bias_act_op(const at::Tensor& x, c10::optional<at::Tensor> bias, int64_t act) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t cols = xc.size(-1), rows = xc.numel() / std::max<int64_t>(cols, 1);
  at::Tensor out = at::empty_like(xc);
  const void* bp = nullptr;
  DType bdt = DType::F32;
  at::Tensor bc;
  if (bias.has_value()) {
    bc = bias->contiguous();
    TORCH_CHECK(bc.numel() == cols, "dlvk.bias_act: bias size");
    bp = bc.data_ptr();
    bdt = to_dtype(bc);
  }
  bias_act(to_dtype(xc), bdt, xc.data_ptr(), bp, out.data_ptr(), rows, cols, (int)act, stream());
  return out;
}

// ---- reductions ----
at::Tensor reduce_op(const at::Tensor& x, int64_t op, double scale) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  auto out = at::empty({}, xc.options().dtype(at::kFloat));
  auto scratch = at::empty({reduce_scratch_floats()}, xc.options().dtype(at::kFloat));
  reduce(to_dtype(xc), xc.data_ptr(), xc.numel(), (int)op, (float)scale, out.data_ptr<float>(),
         scratch.data_ptr<float>(), stream());
  return out;
}

at::Tensor colsum_op(const at::Tensor& x, double scale, c10::optional<at::Tensor> out, bool accumulate,
                     c10::optional<at::ScalarType> out_dtype) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t cols = xc.size(-1), rows = xc.numel() / std::max<int64_t>(cols, 1);
  at::Tensor o = out.has_value() ? *out : at::empty({cols}, xc.options().dtype(out_dtype.value_or(at::kFloat)));
  TORCH_CHECK(o.is_contiguous() && o.numel() == cols, "dlvk.colsum: bad out");
  const int64_t ns = colsum_scratch_floats(rows, cols);
  at::Tensor scratch = ns > 0 ? at::empty({ns}, xc.options().dtype(at::kFloat)) : at::Tensor();
  colsum(to_dtype(xc), to_dtype(o), xc.data_ptr(), rows, cols, (float)scale, o.data_ptr(), accumulate,
         ns > 0 ? scratch.data_ptr<float>() : nullptr, stream());
  return o;
}

at::Tensor rowsum_op(const at::Tensor& x, double scale) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t cols = xc.size(-1), rows = xc.numel() / std::max<int64_t>(cols, 1);
  auto o = at::empty({rows}, xc.options().dtype(at::kFloat));
  rowsum(to_dtype(xc), xc.data_ptr(), rows, cols, (float)scale, o.data_ptr<float>(), stream());
  return o;
}

at::Tensor transpose_op(const at::Tensor& x) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 2 || x.dim() == 3, "dlvk.transpose: 2-D or batched 2-D");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t B = xc.dim() == 3 ? xc.size(0) : 1;
  const int64_t R = xc.size(-2), Cc = xc.size(-1);
  at::Tensor y = xc.dim() == 3 ? at::empty({B, Cc, R}, xc.options()) : at::empty({Cc, R}, xc.options());
  transpose2d(to_dtype(xc), xc.data_ptr(), y.data_ptr(), B, R, Cc, stream());
  return y;
}

at::Tensor permute4_op(const at::Tensor& x, std::vector<int64_t> perm) {
  check_cuda(x, "x");
  TORCH_CHECK(x.dim() == 4 && perm.size() == 4, "dlvk.permute4: 4-D");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  int dims[4], p[4];
  std::vector<int64_t> od(4);
  for (int i = 0; i < 4; ++i) {
    dims[i] = (int)xc.size(i);
    p[i] = (int)perm[i];
  }
  for (int i = 0; i < 4; ++i) od[i] = xc.size(p[i]);
  auto y = at::empty(od, xc.options());
  permute4(to_dtype(xc), xc.data_ptr(), y.data_ptr(), dims, p, stream());
  return y;
}

// ---- softmax / losses ----
at::Tensor softmax_op(const at::Tensor& x, bool log_out) {
  check_cuda(x, "x");
  c10::cuda::CUDAGuard g(x.device());
  auto xc = x.contiguous();
  const int64_t cols = xc.size(-1), rows = xc.numel() / std::max<int64_t>(cols, 1);
  auto y = at::empty_like(xc);
  softmax(to_dtype(xc), xc.data_ptr(), y.data_ptr(), rows, cols, log_out, stream());
  return y;
}

at::Tensor softmax_bwd_op(const at::Tensor& y, const at::Tensor& dy) {
  check_cuda(y, "y");
  c10::cuda::CUDAGuard g(y.device());
  auto yc = y.contiguous(), dyc = dy.contiguous();
  const int64_t cols = yc.size(-1), rows = yc.numel() / std::max<int64_t>(cols, 1);
  auto dx = at::empty_like(yc);
  softmax_bwd(to_dtype(yc), yc.data_ptr(), dyc.data_ptr(), dx.data_ptr(), rows, cols, stream());
  return dx;
}

// Returns (loss_rows [rows] f32, dlogits or empty).  `target` is int32 labels
// [rows] or f32 probabilities [rows, cols].  in_place writes dlogits over the
// logits buffer.
std::vector<at::Tensor> softmax_ce_op(const at::Tensor& logits, const at::Tensor& target, double grad_scale,
                                      bool want_grad, bool in_place) {
  check_cuda(logits, "logits");
  c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.is_contiguous(), "dlvk.softmax_ce: logits must be contiguous");
  const int64_t cols = logits.size(-1), rows = logits.numel() / std::max<int64_t>(cols, 1);
  const int* labels = nullptr;
  const float* probs = nullptr;
  at::Tensor tc;
  if (target.scalar_type() == at::kInt) {
    tc = target.contiguous();
    TORCH_CHECK(tc.numel() == rows, "dlvk.softmax_ce: labels size");
    labels = tc.data_ptr<int>();
  } else {
    tc = target.to(at::kFloat).contiguous();
    TORCH_CHECK(tc.numel() == rows * cols, "dlvk.softmax_ce: target size");
    probs = tc.data_ptr<float>();
  }
  auto loss_rows = at::empty({rows}, logits.options().dtype(at::kFloat));
  at::Tensor dl;
  if (want_grad) dl = in_place ? logits : at::empty_like(logits);
  softmax_cross_entropy(to_dtype(logits), logits.data_ptr(), labels, probs, loss_rows.data_ptr<float>(),
                        want_grad ? dl.data_ptr() : nullptr, rows, cols, (float)grad_scale, stream());
  return {loss_rows, want_grad ? dl : at::Tensor()};
}

at::Tensor sum_scalar_op(const at::Tensor& v, double scale) {
  check_cuda(v, "v");
  TORCH_CHECK(v.scalar_type() == at::kFloat && v.is_contiguous(), "dlvk.sum_scalar: f32 contiguous");
  c10::cuda::CUDAGuard g(v.device());
  auto out = at::empty({}, v.options());
  sum_rows_to_scalar(v.data_ptr<float>(), v.numel(), (float)scale, out.data_ptr<float>(), stream());
  return out;
}

std::vector<at::Tensor> pointwise_loss_op(const at::Tensor& p, const at::Tensor& t, int64_t kind, double loss_scale,
                                          double grad_scale, bool want_grad) {
  check_cuda(p, "p");
  c10::cuda::CUDAGuard g(p.device());
  auto pc = p.contiguous();
  auto tc = t.to(at::kFloat).contiguous();
  TORCH_CHECK(pc.numel() == tc.numel(), "dlvk.pointwise_loss: size mismatch");
  auto out = at::empty({}, pc.options().dtype(at::kFloat));
  auto scratch = at::empty({pointwise_loss_blocks(pc.numel())}, pc.options().dtype(at::kFloat));
  at::Tensor grad = want_grad ? at::empty_like(pc) : at::Tensor();
  pointwise_loss(to_dtype(pc), (int)kind, pc.data_ptr(), tc.data_ptr<float>(), pc.numel(), (float)loss_scale,
                 (float)grad_scale, want_grad ? grad.data_ptr() : nullptr, out.data_ptr<float>(),
                 scratch.data_ptr<float>(), stream());
  return {out, grad};
}

// ---- GEMM ----
// C = act(alpha * A @ B + beta * C + bias + residual).  A: [M,K], [b,M,K] or
// [b,b2,M,K] (any strides; one unit stride per operand for the tensor-core
// path); B likewise [.., K, N].  Transposes and head splits are views.
// fp32 GEMMs on the tensor cores: DLVK_FP32_GEMM = 3xtf32 (default: the
// product split into three TF32 products, error ~1e-6 relative, as fp32
// SIMT), tf32 (one TF32 product, ~1e-3 relative) or simt (CUDA cores
// only).  GEMMs below kTf32MinMacs multiply-adds stay on the SIMT kernel.
constexpr double kTf32MinMacs = 67108864.0;  // 2^26

namespace {
int& fp32_mode_slot() {
  static int mode = [] {
    const char* e = std::getenv("DLVK_FP32_GEMM");
    if (e == nullptr) return 3;
    const std::string v(e);
    return v == "simt" ? 0 : (v == "tf32" ? 1 : 3);
  }();
  return mode;
}
}  // namespace

int fp32_gemm_mode() { return fp32_mode_slot(); }
void set_fp32_gemm_mode(int mode) {
  TORCH_CHECK(mode == 0 || mode == 1 || mode == 3, "dlvk: fp32 GEMM mode is 0 (simt), 1 (tf32) or 3 (3xtf32)");
  fp32_mode_slot() = mode;
}

bool gemm_tf32_ok(const at::Tensor& A, const at::Tensor& B) {
  if (A.scalar_type() != at::kFloat || B.scalar_type() != at::kFloat) return false;
  if (A.dim() != B.dim() || A.dim() < 2 || A.dim() > 4) return false;
  GemmArgs a = fill_args(A, B, A);
  return gemm_tf32_tc_supported(a);
}

namespace {
// hi / lo halves of an fp32 operand with the operand's own strides (a dense
// view such as a transpose keeps its major-ness); other views are split
// from a contiguous copy.
std::pair<at::Tensor, at::Tensor> split_tf32(const at::Tensor& X) {
  at::Tensor src = X.is_non_overlapping_and_dense() ? X : X.contiguous();
  at::Tensor hi = at::empty_strided(src.sizes(), src.strides(), src.options());
  at::Tensor lo = at::empty_strided(src.sizes(), src.strides(), src.options());
  tf32_split(src.data_ptr<float>(), hi.data_ptr<float>(), lo.data_ptr<float>(), src.numel(), stream());
  return {hi, lo};
}

void run_tf32(const GemmArgs& a, int max_ctas, const at::Tensor& like) {
  const int64_t wsf = gemm_tc_workspace_floats(a, max_ctas, DType::F32, true);
  at::Tensor ws = wsf > 0 ? at::empty({wsf}, like.options().dtype(at::kFloat)) : at::Tensor();
  gemm_tf32_tc(DType::F32, a, stream(), device_error_word(), max_ctas, wsf > 0 ? ws.data_ptr<float>() : nullptr, wsf);
}
}  // namespace

// C (fp32) = epilogue(alpha * A B + beta * C) with fp32 A, B on the tensor
// cores.  three_pass: C = alpha Alo Bhi + beta C; C += alpha Ahi Blo;
// C = epilogue(alpha Ahi Bhi + C) -- small terms first, the bias /
// activation / residual / mask only on the last pass.
void gemm_tf32_op(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, const GemmArgs& args, bool three_pass,
                  int max_ctas) {
  if (!three_pass) {
    run_tf32(args, max_ctas, C);
    return;
  }
  auto sa = split_tf32(A);
  auto sb = split_tf32(B);
  GemmArgs lin = fill_args(sa.second, sb.first, C);
  lin.alpha = args.alpha;
  lin.beta = args.beta;
  run_tf32(lin, max_ctas, C);
  lin = fill_args(sa.first, sb.second, C);
  lin.alpha = args.alpha;
  lin.beta = 1.f;
  run_tf32(lin, max_ctas, C);
  GemmArgs last = args;
  const GemmArgs hh = fill_args(sa.first, sb.first, C);
  last.A = hh.A;
  last.B = hh.B;
  last.sam = hh.sam;
  last.sak = hh.sak;
  last.sbk = hh.sbk;
  last.sbn = hh.sbn;
  last.batch_stride_a = hh.batch_stride_a;
  last.batch_stride_b = hh.batch_stride_b;
  last.batch2_stride_a = hh.batch2_stride_a;
  last.batch2_stride_b = hh.batch2_stride_b;
  last.beta = 1.f;
  run_tf32(last, max_ctas, C);
}

GemmArgs fill_args(const at::Tensor& A, const at::Tensor& B, const at::Tensor& C) {
  GemmArgs a;
  const int nd = A.dim();
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.C = C.data_ptr();
  a.M = A.size(-2);
  a.K = A.size(-1);
  a.N = B.size(-1);
  a.sam = A.stride(-2);
  a.sak = A.stride(-1);
  a.sbk = B.stride(-2);
  a.sbn = B.stride(-1);
  a.ldc = C.stride(-2);
  if (nd >= 3) {
    a.batch = A.size(0);
    a.batch_stride_a = A.stride(0);
    a.batch_stride_b = B.stride(0);
    a.batch_stride_c = C.stride(0);
  }
  if (nd == 4) {
    a.batch2 = A.size(1);
    a.batch2_stride_a = A.stride(1);
    a.batch2_stride_b = B.stride(1);
    a.batch2_stride_c = C.stride(1);
  }
  return a;
}

at::Tensor gemm_op(const at::Tensor& A, const at::Tensor& B, c10::optional<at::Tensor> bias, int64_t act,
                   double alpha, double beta, c10::optional<at::Tensor> out, c10::optional<at::ScalarType> out_dtype,
                   int64_t force_path, int64_t max_ctas, c10::optional<at::Tensor> residual,
                   c10::optional<at::Tensor> relu_mask, c10::optional<at::Tensor> colsum_out,
                   double colsum_scale, bool colsum_accumulate, c10::optional<at::Tensor> relu_bits_out,
                   c10::optional<at::Tensor> relu_bits) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "dlvk.gemm: A and B must have the same dtype");
  TORCH_CHECK(A.dim() == B.dim() && A.dim() >= 2 && A.dim() <= 4, "dlvk.gemm: 2-D, 3-D or 4-D operands");
  c10::cuda::CUDAGuard g(A.device());
  const int nd = A.dim();
  for (int i = 0; i < nd - 2; ++i) TORCH_CHECK(A.size(i) == B.size(i), "dlvk.gemm: batch mismatch");
  const int64_t M = A.size(-2), K = A.size(-1), N = B.size(-1);
  TORCH_CHECK(B.size(-2) == K, "dlvk.gemm: inner dims ", K, " vs ", B.size(-2));
  at::Tensor C;
  if (out.has_value()) {
    C = *out;
    TORCH_CHECK(C.dim() == nd && C.size(-1) == N && C.size(-2) == M && C.stride(-1) == 1, "dlvk.gemm: bad out");
  } else {
    auto odt = out_dtype.value_or(A.scalar_type());
    std::vector<int64_t> shp(A.sizes().begin(), A.sizes().end());
    shp.back() = N;
    C = at::empty(shp, A.options().dtype(odt));
    TORCH_CHECK(beta == 0.0, "dlvk.gemm: beta != 0 requires out");
  }
  GemmArgs a = fill_args(A, B, C);
  a.alpha = (float)alpha;
  a.beta = (float)beta;
  at::Tensor bc;
  if (bias.has_value()) {
    bc = bias->contiguous();
    TORCH_CHECK(bc.numel() == N, "dlvk.gemm: bias size");
    a.bias = bc.data_ptr();
    a.bias_dtype = (int)to_dtype(bc);
  }
  if (residual.has_value()) {
    const auto& R = *residual;
    TORCH_CHECK(R.scalar_type() == C.scalar_type() && R.dim() == nd && R.size(-1) == N && R.size(-2) == M &&
                    R.stride(-1) == 1,
                "dlvk.gemm: residual must match the output's dtype/shape with unit column stride");
    a.residual = R.data_ptr();
    a.ldr = R.stride(-2);
    if (nd >= 3) a.batch_stride_r = R.stride(0);
    if (nd == 4) a.batch2_stride_r = R.stride(1);
  }
  if (relu_mask.has_value()) {
    const auto& Mk = *relu_mask;
    TORCH_CHECK(Mk.scalar_type() == C.scalar_type() && Mk.dim() == nd && Mk.size(-1) == N && Mk.size(-2) == M &&
                    Mk.stride(-1) == 1,
                "dlvk.gemm: relu_mask must match the output's dtype/shape with unit column stride");
    a.relu_mask = Mk.data_ptr();
    a.ldm = Mk.stride(-2);
    if (nd >= 3) a.batch_stride_m = Mk.stride(0);
    if (nd == 4) a.batch2_stride_m = Mk.stride(1);
  }
  // ReLU bitmask [M, ceil(N / 32)] int32 words (2-D GEMMs)
  auto bits_arg = [&](const c10::optional<at::Tensor>& t, const char* what) -> at::Tensor {
    if (!t.has_value()) return at::Tensor();
    TORCH_CHECK(nd == 2, "dlvk.gemm: ", what, " needs a 2-D GEMM");
    TORCH_CHECK(t->scalar_type() == at::kInt && t->dim() == 2 && t->size(0) == M && t->size(1) >= (N + 31) / 32 &&
                    t->stride(1) == 1 && t->device() == C.device(),
                "dlvk.gemm: ", what, " must be int32 [M, >= ceil(N / 32)] with unit column stride on C's device");
    a.ldbits = t->stride(0);
    return *t;
  };
  at::Tensor bits_o = bits_arg(relu_bits_out, "relu_bits_out");
  at::Tensor bits_i = bits_arg(relu_bits, "relu_bits");
  if (bits_o.defined()) a.relu_bits_out = reinterpret_cast<uint32_t*>(bits_o.data_ptr<int32_t>());
  if (bits_i.defined()) a.relu_bits = reinterpret_cast<const uint32_t*>(bits_i.data_ptr<int32_t>());
  TORCH_CHECK(!(bits_o.defined() && bits_i.defined()) || bits_o.stride(0) == bits_i.stride(0),
              "dlvk.gemm: relu_bits_out and relu_bits with different row strides");

  a.act = (int)act;
  if (M == 0 || N == 0) return C;
  if (K == 0) {
    // Degenerate: C = act(beta*C + bias + residual).  Rare; do it with ATen.
    TORCH_CHECK(!bits_o.defined() && !bits_i.defined(), "dlvk.gemm: ReLU bitmask with K = 0");
    if (beta == 0.0) C.zero_();
    else C.mul_(beta);
    if (bias.has_value()) C.add_(bc.to(C.scalar_type()));
    if (residual.has_value()) C.add_(*residual);
    if (act == ACT_RELU) C.relu_();
    if (relu_mask.has_value()) C.mul_(relu_mask->gt(0));
    return C;
  }
  const bool tc_ok = A.scalar_type() == at::kBFloat16 && gemm_tc_supported(a) &&
                     (C.scalar_type() == at::kBFloat16 || C.scalar_type() == at::kFloat);
  const bool use_tc = force_path == 1 ? true : (force_path == 2 ? false : tc_ok);
  // colsum_out[n] (+)= colsum_scale * sum over rows of the output: fused into
  // the tensor-core epilogue where its layout allows, else a column-sum pass.
  at::Tensor cs_part;
  if (colsum_out.has_value()) {
    TORCH_CHECK(colsum_out->scalar_type() == at::kFloat && colsum_out->is_contiguous() && colsum_out->numel() == N &&
                    colsum_out->device() == C.device() && nd == 2,
                "dlvk.gemm: colsum_out must be a contiguous fp32 [N] tensor on the output's device (2-D GEMM)");
    if (use_tc && tc_ok && gemm_tc_colsum_ok(to_dtype(C), a)) {
      cs_part = at::empty({(M + 31) / 32 * N}, A.options().dtype(at::kFloat));
      a.colsum = cs_part.data_ptr<float>();
    }
  }
  const int fmode = fp32_gemm_mode();
  const bool tf32_path = A.scalar_type() == at::kFloat && C.scalar_type() == at::kFloat && fmode != 0 &&
                         force_path != 2 && gemm_tf32_tc_supported(a) &&
                         (force_path == 1 || (double)M * N * K * a.batch * a.batch2 >= kTf32MinMacs);
  if (tf32_path) {
    gemm_tf32_op(A, B, C, a, fmode == 3, (int)max_ctas);
  } else if (use_tc) {
    TORCH_CHECK(tc_ok, "dlvk.gemm: tensor-core path requested but not applicable to these operands");
    const int64_t wsf = gemm_tc_workspace_floats(a, (int)max_ctas, to_dtype(C));
    at::Tensor ws = wsf > 0 ? at::empty({wsf}, A.options().dtype(at::kFloat)) : at::Tensor();
    gemm_tc(to_dtype(C), a, stream(), device_error_word(), (int)max_ctas, wsf > 0 ? ws.data_ptr<float>() : nullptr,
            wsf);
  } else {
    if (bits_o.defined()) bits_o.zero_();  // the SIMT kernel sets bits with atomic ORs
    const int64_t swf = gemm_simt_workspace_floats(a);
    at::Tensor sws = swf > 0 ? at::empty({swf}, A.options().dtype(at::kFloat)) : at::Tensor();
    gemm_simt(to_dtype(A), to_dtype(C), a, stream(), swf > 0 ? sws.data_ptr<float>() : nullptr, swf);
  }
  if (colsum_out.has_value()) {
    if (a.colsum != nullptr) {
      colsum_partials(a.colsum, (M + 31) / 32, N, (float)colsum_scale, colsum_out->data_ptr<float>(),
                      colsum_accumulate, stream());
    } else {
      TORCH_CHECK(C.stride(-2) == N, "dlvk.gemm: colsum_out with a strided output needs the fused path");
      const int64_t ns = colsum_scratch_floats(M, N);
      at::Tensor scr = ns > 0 ? at::empty({ns}, A.options().dtype(at::kFloat)) : at::Tensor();
      colsum(to_dtype(C), DType::F32, C.data_ptr(), M, N, (float)colsum_scale, colsum_out->data_ptr<float>(),
             colsum_accumulate, ns > 0 ? scr.data_ptr<float>() : nullptr, stream());
    }
  }
  return C;
}

bool gemm_tc_ok(const at::Tensor& A, const at::Tensor& B) {
  if (A.scalar_type() != at::kBFloat16 || B.scalar_type() != at::kBFloat16) return false;
  if (A.dim() != B.dim() || A.dim() < 2 || A.dim() > 4) return false;
  GemmArgs a = fill_args(A, B, A);
  return gemm_tc_supported(a);
}

// ---- optimizers ----
void optim_advance_op(const at::Tensor& hyper) {
  check_cuda(hyper, "hyper");
  c10::cuda::CUDAGuard g(hyper.device());
  optim_advance(reinterpret_cast<OptimHyper*>(hyper.data_ptr()), stream());
}

void optim_update_op(int64_t kind, const at::Tensor& hyper, const at::Tensor& p, const at::Tensor& grad,
                     c10::optional<at::Tensor> m, c10::optional<at::Tensor> v, c10::optional<at::Tensor> p_bf16,
                     double extra_scale, int64_t max_ctas) {
  check_cuda(p, "p");
  c10::cuda::CUDAGuard g(p.device());
  TORCH_CHECK(p.scalar_type() == at::kFloat && p.is_contiguous(), "dlvk.optim_update: f32 contiguous params");
  TORCH_CHECK(grad.is_contiguous() && grad.numel() == p.numel(), "dlvk.optim_update: grad");
  float* mp = m.has_value() ? m->data_ptr<float>() : nullptr;
  float* vp = v.has_value() ? v->data_ptr<float>() : nullptr;
  if (kind == OPT_ADAM) TORCH_CHECK(mp && vp, "adam needs m and v");
  if (kind == OPT_RMSPROP) TORCH_CHECK(vp, "rmsprop needs v");
  __nv_bfloat16* pb = nullptr;
  if (p_bf16.has_value()) {
    TORCH_CHECK(p_bf16->scalar_type() == at::kBFloat16 && p_bf16->is_contiguous() && p_bf16->numel() == p.numel(),
                "dlvk.optim_update: bf16 copy");
    pb = reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr());
  }
  optim_update((int)kind, reinterpret_cast<const OptimHyper*>(hyper.data_ptr()), p.data_ptr<float>(),
               grad.data_ptr(), to_dtype(grad), mp, vp, pb, p.numel(), (float)extra_scale, stream(), (int)max_ctas);
}

void grad_stats_op(const at::Tensor& g, double scale, double max_norm, const at::Tensor& sumsq,
                   c10::optional<at::Tensor> flag, c10::optional<at::Tensor> clip, bool accumulate,
                   const at::Tensor& scratch, c10::optional<at::Tensor> scale_dev) {
  check_cuda(g, "g");
  c10::cuda::CUDAGuard gd(g.device());
  TORCH_CHECK(g.is_contiguous(), "grad_stats: contiguous grad");
  TORCH_CHECK(scratch.numel() >= grad_stats_scratch_floats(), "grad_stats: scratch too small");
  grad_stats(g.data_ptr(), to_dtype(g), g.numel(), (float)scale, (float)max_norm, sumsq.data_ptr<float>(),
             flag.has_value() ? flag->data_ptr<int>() : nullptr, clip.has_value() ? clip->data_ptr<float>() : nullptr,
             accumulate, scratch.data_ptr<float>(), stream(),
             scale_dev.has_value() ? scale_dev->data_ptr<float>() : nullptr);
}

void scaler_update_op(const at::Tensor& scale, const at::Tensor& good_steps, const at::Tensor& found_inf,
                      double growth, double backoff, int64_t interval, double smin, double smax,
                      c10::optional<at::Tensor> inv_scale) {
  c10::cuda::CUDAGuard g(scale.device());
  scaler_update(scale.data_ptr<float>(), good_steps.data_ptr<int>(), found_inf.data_ptr<int>(), (float)growth,
                (float)backoff, (int)interval, (float)smin, (float)smax,
                inv_scale.has_value() ? inv_scale->data_ptr<float>() : nullptr, stream());
}

int64_t optim_hyper_bytes() { return (int64_t)sizeof(OptimHyper); }

}  // namespace aten
}  // namespace dlvk
