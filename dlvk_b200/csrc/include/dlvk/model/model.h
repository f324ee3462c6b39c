// C++ API: Model / Sequential / ModelTrainer (include/dlvk/model/model.h:
// 15-143 of the reference).
//
// Sequential owns its layers, packs their parameters into flat fp32 buffers
// (reverse registration order, 256-byte aligned slots: the layout the
// Python package uses, so the two produce identical checkpoints), fuses
// Dense + ReLU into one GEMM (whose consumer applies the ReLU backward in
// its dX GEMM) and Conv2D + ReLU into one convolution, and with a trailing
// Softmax trains on the logits with the fused softmax + cross-entropy
// kernel.  save_weights / load_weights write and read `.dlvk` v2 files
// (the framing of the reference's DLVK files, src/training/
// model_persistence.cpp:13-45, with typed tensor records), including the
// optimizer state when one is given.
#pragma once
#include <ATen/core/Generator.h>

#include <functional>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "dlvk/core/cuda_device.h"
#include "dlvk/layers/layers.h"
#include "dlvk/loss/loss_functions.h"
#include "dlvk/optimizers/optimizers.h"
#include "dlvk/tensor/tensor.h"

namespace dlvk {

class Model {
 public:
  virtual ~Model() = default;
  virtual Tensor forward(const Tensor& input) = 0;
  virtual void backward(const Tensor& grad_output) = 0;
  virtual void update_parameters(Optimizer& optimizer) = 0;
  virtual void set_training(bool training) = 0;
  virtual std::string summary() const = 0;
  virtual size_t parameter_count() const = 0;
  virtual void save_weights(const std::string& filepath) const = 0;
  virtual void load_weights(const std::string& filepath) = 0;
};

class Sequential : public Model {
 public:
  explicit Sequential(std::shared_ptr<CudaDevice> device, uint64_t seed = 0);
  ~Sequential() override;
  Sequential(const Sequential&) = delete;
  Sequential& operator=(const Sequential&) = delete;

  // Deep copy (the reference's Sequential::clone, model.h:39-46): same
  // device, seed, step count and training flag, copies of every layer's
  // weights and buffers; dropout layers draw from the copy's own stream
  // state, so the copy's next masks equal the original's.
  std::unique_ptr<Sequential> clone() const;

  void add(std::unique_ptr<ModernLayer> layer);
  void add_layer(std::unique_ptr<ModernLayer> layer) { add(std::move(layer)); }
  void add_dense(size_t input_size, size_t output_size, bool use_bias = true);
  void add_conv2d(size_t in_channels, size_t out_channels, size_t kernel_size, size_t stride = 1,
                  size_t padding = 0);
  void add_maxpool2d(size_t pool_size, size_t stride = 0);
  void add_avgpool2d(size_t pool_size, size_t stride = 0);
  void add_batchnorm1d(size_t num_features);
  void add_batchnorm2d(size_t num_features);
  void add_dropout(float dropout_rate);
  void add_relu();
  void add_sigmoid();
  void add_tanh();
  void add_softmax();
  void add_flatten();

  Tensor forward(const Tensor& input) override;
  // Forward without a trailing Softmax (what the fused loss consumes).
  Tensor forward_logits(const Tensor& input);
  void backward(const Tensor& grad_output) override;
  void update_parameters(Optimizer& optimizer) override;
  void set_training(bool training) override;
  std::string summary() const override;
  size_t parameter_count() const override;
  void save_weights(const std::string& filepath) const override;
  void load_weights(const std::string& filepath) override;
  // Checkpoint with the optimizer state (and restore it).
  void save_weights(const std::string& filepath, const Optimizer* optimizer) const;
  void load_weights(const std::string& filepath, Optimizer* optimizer);

  // One forward / backward / update; returns the loss as a one-element
  // tensor on the model's device (no host synchronisation).
  Tensor train_step(const Tensor& x, const Tensor& y, LossFunction& loss, Optimizer& optimizer);
  void zero_grad();

  size_t size() const { return layers_.size(); }
  ModernLayer& operator[](size_t index) { return *layers_[index]; }
  const ModernLayer& operator[](size_t index) const { return *layers_[index]; }
  const std::vector<std::unique_ptr<ModernLayer>>& layers() const { return layers_; }
  bool has_trailing_softmax() const;
  std::shared_ptr<CudaDevice> device() const { return device_; }

  // Flat buffers (valid after the first forward or build()).
  void build();
  at::Tensor& master() { return master_; }
  at::Tensor& grad() { return grad_; }
  int64_t flat_numel() const { return numel_; }
  std::vector<Parameter*> parameters();
  uint64_t seed() const { return seed_; }
  int64_t step() const { return step_; }
  // All layer tensors with their `.dlvk` record names ("layers.<i>.<name>").
  std::vector<std::pair<std::string, at::Tensor*>> state_tensors() const;
  std::string architecture_json() const;

 private:
  struct Step {
    size_t first, count;
    std::function<Tensor(const Tensor&)> fwd;
  };
  Tensor run(const Tensor& x, size_t upto);
  void make_plan();
  at::Tensor prepare_input(const Tensor& x) const;
  std::string meta_json(const Optimizer* optimizer) const;

  std::shared_ptr<CudaDevice> device_;
  std::vector<std::unique_ptr<ModernLayer>> layers_;
  std::vector<Step> plan_;
  at::Generator gen_;
  uint64_t seed_;
  int64_t step_ = 0;
  int64_t dropout_sites_ = 0;
  bool training_ = true;
  bool built_ = false;
  at::Tensor master_, grad_;
  int64_t numel_ = 0;
  Tensor last_out_;
  size_t last_steps_ = 0;  // plan steps the last forward ran
};

struct TrainingMetrics {
  float loss = 0.0f;
  float accuracy = 0.0f;
  float validation_loss = 0.0f;
  float validation_accuracy = 0.0f;
  size_t epoch = 0;
  size_t batch = 0;
};

class TrainingCallback {
 public:
  virtual ~TrainingCallback() = default;
  virtual void on_train_begin() {}
  virtual void on_train_end() {}
  virtual void on_epoch_begin(size_t /*epoch*/) {}
  virtual void on_epoch_end(size_t /*epoch*/, const TrainingMetrics& /*metrics*/) {}
  virtual void on_batch_begin(size_t /*batch*/) {}
  virtual void on_batch_end(size_t /*batch*/, const TrainingMetrics& /*metrics*/) {}
};

// Mini-batch training loop over in-memory tensors (the reference's
// ModelTrainer, src/model/model.cpp:223-318): batches are row slices, the
// validation split holds out the last rows, metrics are real.
class ModelTrainer {
 public:
  explicit ModelTrainer(Sequential* model);
  void compile(std::unique_ptr<Optimizer> optimizer, std::unique_ptr<LossFunction> loss_function);
  void add_callback(std::unique_ptr<TrainingCallback> callback);
  std::vector<TrainingMetrics> fit(const Tensor& x_train, const Tensor& y_train, size_t epochs,
                                   size_t batch_size = 32, float validation_split = 0.0f, bool verbose = true);
  TrainingMetrics evaluate(const Tensor& x_test, const Tensor& y_test, size_t batch_size = 32);
  Tensor predict(const Tensor& x, size_t batch_size = 32);
  Optimizer* get_optimizer() { return optimizer_.get(); }

 private:
  std::pair<float, float> batch_metrics(const Tensor& x, const Tensor& y);
  Sequential* model_;
  std::unique_ptr<Optimizer> optimizer_;
  std::unique_ptr<LossFunction> loss_;
  std::vector<std::unique_ptr<TrainingCallback>> callbacks_;
};

}  // namespace dlvk
