// C++ API: the layers of the reference's Sequential builder
// (include/dlvk/model/model.h:62-73; dense_layer.h, conv2d_layer.h,
// pooling_layers.h, batch_norm_layers.h, dropout_layer.h, activation.h),
// each with a real forward and backward pass over the framework's kernels.
// Weight layouts are the reference's: Dense W [in, out], Conv2D
// [out, in, k, k].  Initialisation draws from the model's seeded generator
// in the same order and with the same distributions as the Python package,
// so a model built with the same seed starts from the same weights.
#pragma once
#include <ATen/core/Generator.h>

#include "dlvk/layers/modern_layer.h"
#include "dlvk/kernels.h"

namespace dlvk {

enum class ActivationType { ReLU, Sigmoid, Tanh, Softmax };

// Output shape of a k x k window with `stride` and `padding` over an
// [N, C, H, W] or [C, H, W] input: (H + 2 padding - k) / stride + 1 per
// spatial dimension; `channels` replaces C when nonzero.  Throws
// std::invalid_argument for other ranks or a window that does not fit.
std::vector<size_t> window_output_shape(const std::vector<size_t>& input_shape, size_t channels, size_t k,
                                        size_t stride, size_t padding);

class DenseLayer : public ModernLayer {
 public:
  DenseLayer(size_t input_size, size_t output_size, bool use_bias, at::Generator& gen);
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return "Dense"; }
  std::string config_json() const override;

  // Fused execution used by Sequential: `act` in the GEMM epilogue;
  // mask_input: the input is a ReLU output consumed only here, so the dX
  // GEMM applies that ReLU's backward; defer_relu: this layer's own ReLU
  // backward is applied by its consumer.
  Tensor forward_fused(const Tensor& input, int act, bool mask_input, bool defer_relu);

  // Accessors of the reference's dense_layer.h:31-32: views of the fp32
  // masters (W [in, out]); an undefined Tensor when built without a bias.
  Tensor get_weights() const { return Tensor(weight_->master); }
  Tensor get_bias() const { return bias_ ? Tensor(bias_->master) : Tensor(); }

  size_t input_size, output_size;

 private:
  Parameter* weight_ = nullptr;
  Parameter* bias_ = nullptr;
  at::Tensor x_, y_;
  std::vector<int64_t> in_shape_;
  int act_ = ACT_NONE;
  bool mask_input_ = false, relu_here_ = false;
};

class ActivationLayer : public ModernLayer {
 public:
  explicit ActivationLayer(ActivationType type) : type_(type) {}
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override;
  std::string config_json() const override;
  ActivationType activation() const { return type_; }
  ActivationType get_activation_type() const { return type_; }

 private:
  ActivationType type_;
  at::Tensor saved_;
};

class Conv2DLayer : public ModernLayer {
 public:
  Conv2DLayer(size_t in_channels, size_t out_channels, size_t kernel_size, size_t stride, size_t padding,
              at::Generator& gen);
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return "Conv2D"; }
  std::string config_json() const override;
  Tensor forward_fused(const Tensor& input, bool relu);

  // Accessors of the reference's conv2d_layer.h:40-52 (W [out, in, k, k]).
  Tensor get_weights() const { return Tensor(weight_->master); }
  Tensor get_bias() const { return bias_ ? Tensor(bias_->master) : Tensor(); }
  size_t get_in_channels() const { return in_channels; }
  size_t get_out_channels() const { return out_channels; }
  size_t get_kernel_height() const { return kernel_size; }
  size_t get_kernel_width() const { return kernel_size; }
  std::vector<size_t> compute_output_shape(const std::vector<size_t>& input_shape) const {
    return window_output_shape(input_shape, out_channels, kernel_size, stride, padding);
  }

  size_t in_channels, out_channels, kernel_size, stride, padding;

 private:
  Parameter* weight_ = nullptr;
  Parameter* bias_ = nullptr;
  at::Tensor x_, y_;
  bool relu_ = false;
};

class MaxPool2DLayer : public ModernLayer {
 public:
  MaxPool2DLayer(size_t pool_size, size_t stride) : pool_size(pool_size), stride(stride ? stride : pool_size) {}
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return "MaxPool2D"; }
  std::string config_json() const override;
  // Accessors of the reference's pooling_layers.h:34-38 (square windows).
  size_t get_pool_height() const { return pool_size; }
  size_t get_pool_width() const { return pool_size; }
  std::vector<size_t> compute_output_shape(const std::vector<size_t>& input_shape) const {
    return window_output_shape(input_shape, 0, pool_size, stride, 0);
  }
  size_t pool_size, stride;

 private:
  at::Tensor idx_;
  int64_t H_ = 0, W_ = 0;
};

class AvgPool2DLayer : public ModernLayer {
 public:
  AvgPool2DLayer(size_t pool_size, size_t stride) : pool_size(pool_size), stride(stride ? stride : pool_size) {}
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return "AvgPool2D"; }
  std::string config_json() const override;
  size_t get_pool_height() const { return pool_size; }
  size_t get_pool_width() const { return pool_size; }
  std::vector<size_t> compute_output_shape(const std::vector<size_t>& input_shape) const {
    return window_output_shape(input_shape, 0, pool_size, stride, 0);
  }
  size_t pool_size, stride;

 private:
  int64_t H_ = 0, W_ = 0;
};

// BatchNorm over [N, C] (1-D) or [N, C, H, W] (2-D): biased batch variance,
// running = (1 - m) running + m batch with m = 0.1 (the reference's CPU
// convention, src/layers/batch_norm_layers.cpp:65-116).
class BatchNormLayer : public ModernLayer {
 public:
  BatchNormLayer(size_t num_features, bool two_d, double momentum = 0.1, double eps = 1e-5);
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return two_d_ ? "BatchNorm2D" : "BatchNorm1D"; }
  std::string config_json() const override;
  // Accessors of the reference's batch_norm_layers.h:39-46.  The getters
  // return views; the setters copy into the existing tensors, which stay
  // the model's packed views.
  Tensor get_gamma() const { return Tensor(gamma_->master); }
  Tensor get_beta() const { return Tensor(beta_->master); }
  Tensor get_running_mean() const { return Tensor(running_mean); }
  Tensor get_running_var() const { return Tensor(running_var); }
  void set_gamma(const Tensor& g) { copy_into(gamma_->master, g, "gamma"); }
  void set_beta(const Tensor& b) { copy_into(beta_->master, b, "beta"); }
  void set_running_mean(const Tensor& m) { copy_into(running_mean, m, "running_mean"); }
  void set_running_var(const Tensor& v) { copy_into(running_var, v, "running_var"); }
  size_t num_features;
  double momentum, eps;
  at::Tensor running_mean, running_var;

 protected:
  std::vector<std::pair<std::string, at::Tensor*>> buffers() override;

 private:
  static void copy_into(at::Tensor& dst, const Tensor& src, const char* what);
  bool two_d_;
  Parameter* gamma_ = nullptr;
  Parameter* beta_ = nullptr;
  at::Tensor x_, mean_, rstd_;
};

// Inverted dropout with a counter-based Philox mask keyed by (model seed,
// dropout site, model step): the same mask on CPU and GPU.
class DropoutLayer : public ModernLayer {
 public:
  DropoutLayer(float rate, int64_t site, const uint64_t* seed, const int64_t* step)
      : rate(rate), site_(site), seed_(seed), step_(step) {}
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override;
  std::string type_name() const override { return "Dropout"; }
  std::string config_json() const override;
  float get_dropout_rate() const { return rate; }
  // Throws std::invalid_argument outside [0, 1).
  void set_dropout_rate(float r);
  float rate;

 private:
  int64_t site_;
  const uint64_t* seed_;
  const int64_t* step_;
  int64_t used_step_ = 0;
};

class FlattenLayer : public ModernLayer {
 public:
  Tensor forward(const Tensor& input) override;
  Tensor backward(const Tensor& grad_output) override;
  std::unique_ptr<ModernLayer> clone() const override { return std::make_unique<FlattenLayer>(*this); }
  std::string type_name() const override { return "Flatten"; }

 private:
  std::vector<int64_t> in_shape_;
};

}  // namespace dlvk
