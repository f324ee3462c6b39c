// C++ API: optimizers (include/dlvk/optimizers/optimizers.h:11-155 of the
// reference): SGD with momentum, Adam, RMSprop.
//
// An optimizer keeps its state (Adam m / v, SGD momentum, RMSprop square
// average) as flat fp32 buffers parallel to a model's flat parameter buffer
// and updates all parameters with one kernel launch (optim.cu) that reads
// its hyper-parameters from a small device block.  Adam applies the bias
// corrections 1/(1 - beta^t) that the reference shader documents
// (shaders/adam_update.comp:27-28) and advances its step once per step()
// (the reference counted it twice, src/optimizers/adam.cpp:18,37).
// Hyper-parameters are doubles, as in the Python package, so both front ends
// compute the same update.
#pragma once
#include <ATen/ATen.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace dlvk {

class ModernLayer;
class Sequential;
struct Parameter;

class Optimizer {
 public:
  Optimizer(int kind, double lr, double beta1, double beta2, double eps, double momentum, double alpha,
            double weight_decay);
  virtual ~Optimizer();

  virtual std::string name() const = 0;
  void set_learning_rate(double lr);
  double get_learning_rate() const { return lr_; }
  void set_lr(double lr) { set_learning_rate(lr); }
  double get_lr() const { return lr_; }

  // Gradient clipping (the reference's optimizers.h:41-45), applied by
  // step() / update() before the update: by norm, the gradients are scaled
  // by min(1, max_norm / ||g||) with the norm over the model's whole
  // gradient buffer; by value, every element is clamped to [min, max]
  // (in place, so the model's gradient buffer holds the clamped values).
  void set_grad_clip_norm(double max_norm);
  void set_grad_clip_value(double min_val, double max_val);
  void disable_grad_clipping();

  // One update of every parameter of `model` (advances the step counter).
  void step(Sequential& model);
  // Reference interface: update one layer's parameters.
  void update(ModernLayer* layer);

  // State for `.dlvk` checkpoints: flat buffers ("optim.m", "optim.v") and
  // the metadata object (keys sorted).
  std::vector<std::pair<std::string, at::Tensor*>> state_tensors(const Sequential& model);
  std::string state_meta_json(const Sequential& model) const;
  // Restores the step count and learning rate from that metadata object.
  void load_state_meta(const Sequential& model, int64_t step, double lr);
  int64_t step_count(const Sequential& model) const;

  struct State;

 protected:
  State& state(const Sequential& model);
  const State* find_state(const Sequential& model) const;
  void advance(State& st);
  void update_range(State& st, at::Tensor& master, at::Tensor& grad, int64_t start, int64_t end);
  void prepare_grads(State& st, at::Tensor& grad);

  int kind_;
  double lr_, beta1_, beta2_, eps_, momentum_, alpha_, weight_decay_;
  bool bias_correction_ = true;
  bool use_clip_norm_ = false, use_clip_value_ = false;
  double clip_norm_ = 0.0, clip_min_ = 0.0, clip_max_ = 0.0;
  std::map<const void*, std::unique_ptr<State>> states_;
};

class SGD : public Optimizer {
 public:
  explicit SGD(double learning_rate = 0.01, double momentum = 0.0, double weight_decay = 0.0);
  std::string name() const override { return "SGD"; }
};

class Adam : public Optimizer {
 public:
  explicit Adam(double learning_rate = 0.001, double beta1 = 0.9, double beta2 = 0.999, double epsilon = 1e-8,
                double weight_decay = 0.0);
  std::string name() const override { return "Adam"; }
};

class RMSprop : public Optimizer {
 public:
  explicit RMSprop(double learning_rate = 0.01, double alpha = 0.99, double epsilon = 1e-8);
  std::string name() const override { return "RMSprop"; }
};

}  // namespace dlvk
