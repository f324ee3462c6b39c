// C++ API: loss functions.  Formulas restate the Python package's losses
// (dlvk_b200/losses.py), which keep the reference's CPU definitions
// (src/loss/loss_functions.cpp:59-238): CE = -sum t log(p + 1e-8) / B on
// probabilities, MSE = mean (p - t)^2, BCE with clamped probabilities.
#include "dlvk/loss/loss_functions.h"

#include "dispatch.h"
#include "dlvk/kernels.h"

namespace dlvk {

namespace {
// Class ids ([rows] integers) or probabilities, as a [rows, cols] fp32 tensor.
at::Tensor to_probs(const at::Tensor& t, int64_t cols) {
  if (t.is_floating_point()) return t.to(at::kFloat);
  return at::one_hot(t.reshape({-1}).to(at::kLong), cols).to(at::kFloat);
}
std::shared_ptr<Tensor> wrap(at::Tensor t, const Tensor& like) { return std::make_shared<Tensor>(std::move(t), like.device()); }
}  // namespace

std::pair<Tensor, Tensor> LossFunction::value_and_grad(const Tensor& predictions, const Tensor& targets) {
  auto p = std::make_shared<Tensor>(predictions);
  auto t = std::make_shared<Tensor>(targets);
  return {*forward(p, t), *backward(p, t)};
}

std::shared_ptr<Tensor> CrossEntropyLoss::forward(const std::shared_ptr<Tensor>& pred,
                                                  const std::shared_ptr<Tensor>& targets) {
  at::Tensor p = pred->data().to(at::kFloat);
  at::Tensor p2 = p.reshape({-1, p.size(-1)});
  at::Tensor t = to_probs(targets->data().to(p.device()), p2.size(1)).reshape(p2.sizes());
  return wrap(-(t * at::log(p2 + 1e-8)).sum() / (double)p2.size(0), *pred);
}

std::shared_ptr<Tensor> CrossEntropyLoss::backward(const std::shared_ptr<Tensor>& pred,
                                                   const std::shared_ptr<Tensor>& targets) {
  const at::Tensor& p = pred->data();
  at::Tensor p2 = p.reshape({-1, p.size(-1)}).to(at::kFloat);
  at::Tensor t = to_probs(targets->data().to(p.device()), p2.size(1)).reshape(p2.sizes());
  return wrap((-t / (p2 + 1e-8) / (double)p2.size(0)).to(p.scalar_type()).reshape(p.sizes()), *pred);
}

std::pair<Tensor, Tensor> CrossEntropyLoss::value_and_grad_from_logits(const Tensor& logits, const Tensor& targets) {
  const at::Tensor& out = logits.data();
  const int64_t rows = out.numel() / out.size(-1);
  at::Tensor tgt = targets.data().to(out.device());
  if (!tgt.is_floating_point()) tgt = tgt.to(at::kInt);
  auto r = api::softmax_ce(out.reshape({rows, out.size(-1)}),
                           tgt.is_floating_point() ? tgt.reshape({rows, -1}) : tgt.reshape({rows}), 1.0 / (double)rows);
  at::Tensor loss = api::sum_scalar(r.first, 1.0 / (double)rows);
  return {Tensor(loss, logits.device()), Tensor(r.second.reshape(out.sizes()), logits.device())};
}

std::shared_ptr<Tensor> MeanSquaredError::forward(const std::shared_ptr<Tensor>& pred,
                                                  const std::shared_ptr<Tensor>& targets) {
  const at::Tensor& p = pred->data();
  auto r = api::pointwise_loss(p, targets->data().to(p.device()), LOSS_MSE, 1.0 / (double)p.numel(), 0.0, false);
  return wrap(r.first, *pred);
}

std::shared_ptr<Tensor> MeanSquaredError::backward(const std::shared_ptr<Tensor>& pred,
                                                   const std::shared_ptr<Tensor>& targets) {
  const at::Tensor& p = pred->data();
  const double s = 1.0 / (double)p.numel();
  return wrap(api::pointwise_loss(p, targets->data().to(p.device()), LOSS_MSE, s, s, true).second, *pred);
}

std::shared_ptr<Tensor> BinaryCrossEntropyLoss::forward(const std::shared_ptr<Tensor>& pred,
                                                        const std::shared_ptr<Tensor>& targets) {
  const at::Tensor& p = pred->data();
  auto r = api::pointwise_loss(p, targets->data().to(p.device()), LOSS_BCE, 1.0 / (double)p.numel(), 0.0, false);
  return wrap(r.first, *pred);
}

std::shared_ptr<Tensor> BinaryCrossEntropyLoss::backward(const std::shared_ptr<Tensor>& pred,
                                                         const std::shared_ptr<Tensor>& targets) {
  const at::Tensor& p = pred->data();
  const double s = 1.0 / (double)p.numel();
  return wrap(api::pointwise_loss(p, targets->data().to(p.device()), LOSS_BCE, s, s, true).second, *pred);
}

}  // namespace dlvk
