// C++ API: loss functions (include/dlvk/loss/loss_functions.h of the
// reference).  forward() returns the mean loss as a one-element tensor and
// backward() its gradient with respect to the predictions.  CrossEntropy
// takes probabilities (the output of a trailing softmax) with the
// reference's CPU formula; a Sequential whose last layer is Softmax uses
// value_and_grad_from_logits() instead, the fused softmax + cross-entropy
// kernel on the logits, which is the numerically stable equivalent.
#pragma once
#include <memory>
#include <utility>

#include "dlvk/tensor/tensor.h"

namespace dlvk {

class LossFunction {
 public:
  virtual ~LossFunction() = default;
  virtual std::shared_ptr<Tensor> forward(const std::shared_ptr<Tensor>& predictions,
                                          const std::shared_ptr<Tensor>& targets) = 0;
  virtual std::shared_ptr<Tensor> backward(const std::shared_ptr<Tensor>& predictions,
                                           const std::shared_ptr<Tensor>& targets) = 0;
  // (loss, dloss/dpredictions) in one call.
  virtual std::pair<Tensor, Tensor> value_and_grad(const Tensor& predictions, const Tensor& targets);
  virtual bool fuses_softmax() const { return false; }
};

class MeanSquaredError : public LossFunction {
 public:
  std::shared_ptr<Tensor> forward(const std::shared_ptr<Tensor>& predictions,
                                  const std::shared_ptr<Tensor>& targets) override;
  std::shared_ptr<Tensor> backward(const std::shared_ptr<Tensor>& predictions,
                                   const std::shared_ptr<Tensor>& targets) override;
};

class CrossEntropyLoss : public LossFunction {
 public:
  std::shared_ptr<Tensor> forward(const std::shared_ptr<Tensor>& predictions,
                                  const std::shared_ptr<Tensor>& targets) override;
  std::shared_ptr<Tensor> backward(const std::shared_ptr<Tensor>& predictions,
                                   const std::shared_ptr<Tensor>& targets) override;
  // Fused softmax + cross-entropy from logits; targets are class ids
  // (integer tensor) or probabilities.  Loss is the batch mean.
  std::pair<Tensor, Tensor> value_and_grad_from_logits(const Tensor& logits, const Tensor& targets);
  bool fuses_softmax() const override { return true; }
};

class BinaryCrossEntropyLoss : public LossFunction {
 public:
  explicit BinaryCrossEntropyLoss(float epsilon = 1e-7f) : epsilon_(epsilon) {}
  std::shared_ptr<Tensor> forward(const std::shared_ptr<Tensor>& predictions,
                                  const std::shared_ptr<Tensor>& targets) override;
  std::shared_ptr<Tensor> backward(const std::shared_ptr<Tensor>& predictions,
                                   const std::shared_ptr<Tensor>& targets) override;

 private:
  float epsilon_;
};

}  // namespace dlvk
