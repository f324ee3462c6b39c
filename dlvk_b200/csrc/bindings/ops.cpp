// PyTorch bindings of the dlvk_b200 kernels (module dlvk_b200._C).
// Every op launches on the current CUDA stream of the tensors' device, takes
// strided views where the kernel supports them, and allocates outputs through
// PyTorch's caching allocator (so the ops are CUDA-graph capturable).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "dlvk/kernels.h"
#include "bind_common.h"
#include "dlvk/aten_ops.h"

namespace dlvk {
namespace bind {
using namespace ::dlvk::aten;

void register_ops(py::module& m) {
  m.def("unary", &unary_op, py::arg("x"), py::arg("op"), py::arg("a") = 0.0, py::arg("b") = 0.0,
        py::arg("out") = py::none(), py::arg("out_dtype") = py::none());
  m.def("binary", &binary_op, py::arg("x"), py::arg("y"), py::arg("op"), py::arg("out") = py::none());
  m.def("bias_act", &bias_act_op, py::arg("x"), py::arg("bias") = py::none(), py::arg("act") = 6);
  m.def("reduce", &reduce_op, py::arg("x"), py::arg("op") = 0, py::arg("scale") = 1.0);
  m.def("colsum", &colsum_op, py::arg("x"), py::arg("scale") = 1.0, py::arg("out") = py::none(),
        py::arg("accumulate") = false, py::arg("out_dtype") = py::none());
  m.def("rowsum", &rowsum_op, py::arg("x"), py::arg("scale") = 1.0);
  m.def("transpose", &transpose_op);
  m.def("permute4", &permute4_op);
  m.def("softmax", &softmax_op, py::arg("x"), py::arg("log") = false);
  m.def("softmax_bwd", &softmax_bwd_op);
  m.def("softmax_ce", &softmax_ce_op, py::arg("logits"), py::arg("target"), py::arg("grad_scale") = 1.0,
        py::arg("want_grad") = true, py::arg("in_place") = false);
  m.def("sum_scalar", &sum_scalar_op, py::arg("v"), py::arg("scale") = 1.0);
  m.def("pointwise_loss", &pointwise_loss_op);
  m.def("gemm", &gemm_op, py::arg("A"), py::arg("B"), py::arg("bias") = py::none(), py::arg("act") = 0,
        py::arg("alpha") = 1.0, py::arg("beta") = 0.0, py::arg("out") = py::none(), py::arg("out_dtype") = py::none(),
        py::arg("force_path") = 0, py::arg("max_ctas") = 0, py::arg("residual") = py::none(),
        py::arg("relu_mask") = py::none(), py::arg("colsum_out") = py::none(), py::arg("colsum_scale") = 1.0,
        py::arg("colsum_accumulate") = false, py::arg("relu_bits_out") = py::none(),
        py::arg("relu_bits") = py::none());
  m.def("gemm_tc_ok", &gemm_tc_ok);
  m.def("gemm_tf32_ok", &gemm_tf32_ok);
  m.def("set_fp32_gemm_mode", &set_fp32_gemm_mode);
  m.def("fp32_gemm_mode", &fp32_gemm_mode);
  m.def("optim_advance", &optim_advance_op);
  m.def("optim_update", &optim_update_op, py::arg("kind"), py::arg("hyper"), py::arg("p"), py::arg("grad"),
        py::arg("m") = py::none(), py::arg("v") = py::none(), py::arg("p_bf16") = py::none(),
        py::arg("extra_scale") = 1.0, py::arg("max_ctas") = 0);
  m.def("gemm_set_pair", [](bool on) { gemm_tc_set_pair(on); });
  m.def("gemm_set_wide", [](int64_t mode) { gemm_tc_set_wide((int)mode); });
  m.def("gemm_set_tiling", [](int64_t bn, int64_t splits, int64_t pair) {
    gemm_tc_set_tiling((int)bn, (int)splits, (int)pair);
  }, py::arg("bn") = 0, py::arg("splits") = 0, py::arg("pair") = -1);
  m.def(
      "gemm_plan",
      [](const at::Tensor& A, const at::Tensor& B, bool out_f32, int64_t max_ctas) {
        GemmArgs a = fill_args(A, B, A);
        a.ldc = B.size(-1);
        int bn = 0, sp = 0, pr = 0;
        gemm_tc_plan(out_f32 ? DType::F32 : DType::BF16, a, (int)max_ctas, &bn, &sp, &pr);
        return py::make_tuple(bn, sp, pr != 0);
      },
      py::arg("A"), py::arg("B"), py::arg("out_f32") = false, py::arg("max_ctas") = 0);
  m.def("gemm_pair_enabled", []() { return gemm_tc_pair_enabled(); });
  m.def("grad_stats", &grad_stats_op, py::arg("g"), py::arg("scale"), py::arg("max_norm"), py::arg("sumsq"),
        py::arg("flag"), py::arg("clip"), py::arg("accumulate"), py::arg("scratch"), py::arg("scale_dev") = py::none());
  m.def("step_metrics", [](const at::Tensor& logits, c10::optional<at::Tensor> labels, c10::optional<at::Tensor> probs,
                           c10::optional<at::Tensor> loss, c10::optional<at::Tensor> loss_sum,
                           c10::optional<at::Tensor> correct, double loss_weight) {
    check_cuda(logits, "logits");
    TORCH_CHECK(logits.is_contiguous() && logits.dim() >= 1, "step_metrics: contiguous logits");
    const int cols = (int)logits.size(-1);
    const int64_t rows = cols ? logits.numel() / cols : 0;
    const int* lp = nullptr;
    const float* pp = nullptr;
    if (labels.has_value()) {
      TORCH_CHECK(labels->scalar_type() == at::kInt && labels->numel() == rows, "step_metrics: int32 labels [rows]");
      lp = labels->data_ptr<int>();
    }
    if (probs.has_value()) {
      TORCH_CHECK(probs->scalar_type() == at::kFloat && probs->numel() == rows * cols && probs->is_contiguous(),
                  "step_metrics: fp32 probs [rows, cols]");
      pp = probs->data_ptr<float>();
    }
    c10::cuda::CUDAGuard g(logits.device());
    step_metrics(to_dtype(logits), logits.data_ptr(), rows, cols, lp, pp,
                 loss.has_value() ? loss->data_ptr<float>() : nullptr,
                 loss_sum.has_value() ? loss_sum->data_ptr<float>() : nullptr,
                 correct.has_value() ? reinterpret_cast<unsigned long long*>(correct->data_ptr<int64_t>()) : nullptr,
                 (float)loss_weight, stream());
  }, py::arg("logits"), py::arg("labels") = py::none(), py::arg("probs") = py::none(), py::arg("loss") = py::none(),
     py::arg("loss_sum") = py::none(), py::arg("correct") = py::none(), py::arg("loss_weight") = 1.0);
  m.def("scale_by_device_scalar", [](const at::Tensor& x, const at::Tensor& s) {
    check_cuda(x, "x");
    TORCH_CHECK(x.is_contiguous() && s.scalar_type() == at::kFloat && s.is_cuda(), "scale_by_device_scalar: args");
    c10::cuda::CUDAGuard g(x.device());
    scale_by_device_scalar(to_dtype(x), x.data_ptr(), x.numel(), s.data_ptr<float>(), stream());
  });
  m.def("regularize", [](const at::Tensor& w, const at::Tensor& g, double l1, double l2, double ll1, double ll2,
                         c10::optional<at::Tensor> loss_out, c10::optional<at::Tensor> gscale) {
    check_cuda(w, "w");
    check_cuda(g, "g");
    TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous() && g.is_contiguous() && g.numel() == w.numel(),
                "regularize: w fp32 contiguous, g same numel");
    c10::cuda::CUDAGuard gd(w.device());
    regularize(w.data_ptr<float>(), g.data_ptr(), to_dtype(g), w.numel(), (float)l1, (float)l2, (float)ll1, (float)ll2,
               loss_out.has_value() ? loss_out->data_ptr<float>() : nullptr, stream(),
               gscale.has_value() ? gscale->data_ptr<float>() : nullptr);
  }, py::arg("w"), py::arg("g"), py::arg("l1"), py::arg("l2"), py::arg("ll1"), py::arg("ll2"),
     py::arg("loss_out") = py::none(),
     py::arg("gscale") = py::none());
  m.def("grad_stats_scratch_floats", &grad_stats_scratch_floats);
  m.def("scaler_update", &scaler_update_op);
  m.def("optim_hyper_bytes", &optim_hyper_bytes);
  m.def("memset_zero", [](const at::Tensor& t) {
    check_cuda(t, "t");
    TORCH_CHECK(t.is_contiguous(), "memset_zero: contiguous tensor");
    c10::cuda::CUDAGuard g(t.device());
    DLVK_CUDA_CHECK(cudaMemsetAsync(t.data_ptr(), 0, t.numel() * t.element_size(), stream()));
  });
  m.def("counter_add", [](const at::Tensor& c, int64_t delta) {
    check_cuda(c, "counter");
    TORCH_CHECK(c.scalar_type() == at::kLong, "counter must be int64");
    c10::cuda::CUDAGuard g(c.device());
    counter_add(c.data_ptr<int64_t>(), delta, stream());
  });
  m.def("launch_count", []() { return (int64_t)launch_count(); });
  m.def("read_device_error", [](bool clear) { return (int64_t)read_device_error(clear); }, py::arg("clear") = true);
}

}  // namespace bind
}  // namespace dlvk
