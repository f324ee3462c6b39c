// C++ API: layer implementations.  Each forward / backward restates the
// Python package's autograd function of the same layer (dlvk_b200/ops/
// functional.py: DenseFn, ActivationFn, SoftmaxFn, Conv2dFn, MaxPoolFn,
// AvgPoolFn, BatchNormFn, DropoutFn) with explicit saved tensors instead of
// autograd, and issues the same kernels in the same order.
#include "dlvk/layers/layers.h"

#include <algorithm>
#include <cctype>
#include <cmath>
#include <sstream>
#include <stdexcept>

#include "dispatch.h"
#include "dlvk/optimizers/optimizers.h"
#include "json_util.h"

namespace dlvk {

// ---------------------------------------------------------------- Parameter / ModernLayer
int64_t Parameter::numel() const {
  int64_t n = 1;
  for (auto d : shape) n *= d;
  return n;
}

bool Parameter::take_accumulate() {
  const bool acc = !fresh;
  fresh = false;
  return acc;
}

Parameter& ModernLayer::add_param(const std::string& name, at::Tensor init) {
  auto p = std::make_unique<Parameter>();
  std::string prefix = type_name();
  std::transform(prefix.begin(), prefix.end(), prefix.begin(), [](unsigned char c) { return std::tolower(c); });
  p->name = prefix + "." + name;
  p->shape = std::vector<int64_t>(init.sizes().begin(), init.sizes().end());
  p->master = init.to(at::kFloat).contiguous();
  params_.push_back(std::move(p));
  return *params_.back();
}

ModernLayer::ModernLayer(const ModernLayer& other)
    : output_shape(other.output_shape), need_input_grad(other.need_input_grad), training_(other.training_) {
  for (const auto& q : other.params_) {
    auto p = std::make_unique<Parameter>();
    p->name = q->name;
    p->shape = q->shape;
    p->master = q->master.clone().contiguous();
    params_.push_back(std::move(p));
  }
}

std::vector<Parameter*> ModernLayer::parameters() {
  std::vector<Parameter*> out;
  for (auto& p : params_) out.push_back(p.get());
  return out;
}

std::vector<std::pair<std::string, at::Tensor*>> ModernLayer::state_tensors() {
  std::vector<std::pair<std::string, at::Tensor*>> out;
  for (auto& p : params_) out.emplace_back(p->name, &p->master);
  for (auto& b : buffers()) out.push_back(b);
  return out;
}

size_t ModernLayer::parameter_count() const {
  size_t n = 0;
  for (const auto& p : params_) n += (size_t)p->numel();
  return n;
}

void ModernLayer::update_parameters(Optimizer& optimizer) { optimizer.update(this); }

LayerInfo ModernLayer::get_layer_info() const {
  LayerInfo info;
  info.type = type_name();
  std::string s;
  for (size_t i = 0; i < output_shape.size(); ++i) s += (i ? "x" : "") + std::to_string(output_shape[i]);
  info.output_shape_str = s.empty() ? "?" : s;
  info.parameter_count = parameter_count();
  info.trainable = info.parameter_count > 0;
  return info;
}

std::string ModernLayer::config_json() const { return "{\"type\":" + json::str(type_name()) + "}"; }

void ModernLayer::save_weights(std::ofstream& f) const {
  auto self = const_cast<ModernLayer*>(this)->state_tensors();
  const uint32_t n = (uint32_t)self.size();
  f.write(reinterpret_cast<const char*>(&n), 4);
  for (auto& kv : self) {
    at::Tensor c = kv.second->to(c10::kCPU, at::kFloat).contiguous();
    const uint64_t nb = (uint64_t)c.numel() * 4;
    f.write(reinterpret_cast<const char*>(&nb), 8);
    f.write(reinterpret_cast<const char*>(c.data_ptr<float>()), (std::streamsize)nb);
  }
}

void ModernLayer::load_weights(std::ifstream& f) {
  auto self = state_tensors();
  uint32_t n = 0;
  f.read(reinterpret_cast<char*>(&n), 4);
  TORCH_CHECK(f && n == self.size(), "dlvk: ", type_name(), " expects ", self.size(), " tensors, stream has ", n);
  for (auto& kv : self) {
    uint64_t nb = 0;
    f.read(reinterpret_cast<char*>(&nb), 8);
    TORCH_CHECK(f && nb == (uint64_t)kv.second->numel() * 4, "dlvk: ", kv.first, ": byte count mismatch");
    at::Tensor host = at::empty(kv.second->sizes(), at::kFloat);
    f.read(reinterpret_cast<char*>(host.data_ptr<float>()), (std::streamsize)nb);
    kv.second->copy_(host);
  }
}

namespace {
std::vector<int64_t> sizes_of(const at::Tensor& t) { return std::vector<int64_t>(t.sizes().begin(), t.sizes().end()); }
at::Tensor flat2(const at::Tensor& t) { return t.reshape({-1, t.size(-1)}); }
}  // namespace

// ---------------------------------------------------------------- Dense
DenseLayer::DenseLayer(size_t in, size_t out, bool use_bias, at::Generator& gen) : input_size(in), output_size(out) {
  const double std = std::sqrt(2.0 / (double)(in + out));
  weight_ = &add_param("weight", at::randn({(int64_t)in, (int64_t)out}, gen) * std);
  if (use_bias) bias_ = &add_param("bias", at::zeros({(int64_t)out}));
}

std::unique_ptr<ModernLayer> DenseLayer::clone() const {
  auto c = std::make_unique<DenseLayer>(*this);
  c->weight_ = c->params_[0].get();
  c->bias_ = c->params_.size() > 1 ? c->params_[1].get() : nullptr;
  return c;
}

std::string DenseLayer::config_json() const {
  return "{\"activation\":null,\"input_size\":" + std::to_string(input_size) +
         ",\"output_size\":" + std::to_string(output_size) + ",\"type\":\"Dense\",\"use_bias\":" +
         (bias_ ? "true" : "false") + "}";
}

Tensor DenseLayer::forward(const Tensor& input) { return forward_fused(input, ACT_NONE, false, false); }

Tensor DenseLayer::forward_fused(const Tensor& input, int act, bool mask_input, bool defer_relu) {
  at::Tensor x = input.data();
  if (x.dim() > 2 && x.size(-1) != (int64_t)input_size) x = x.reshape({x.size(0), -1});
  in_shape_ = sizes_of(x);
  at::Tensor x2 = flat2(x);
  at::Tensor y = api::gemm(x2, weight_->master, bias_ ? c10::optional<at::Tensor>(bias_->master) : c10::nullopt, act);
  act_ = act;
  mask_input_ = mask_input;
  relu_here_ = act == ACT_RELU && !defer_relu;
  if (training_) {
    x_ = x2;
    y_ = relu_here_ ? y : at::Tensor();
  }
  std::vector<int64_t> os(in_shape_.begin(), in_shape_.end() - 1);
  os.push_back((int64_t)output_size);
  return Tensor(y.reshape(os), input.device());
}

Tensor DenseLayer::backward(const Tensor& grad_output) {
  TORCH_CHECK(x_.defined(), "dlvk: Dense backward needs a training-mode forward");
  at::Tensor g2 = flat2(grad_output.data());
  if (g2.scalar_type() != x_.scalar_type()) g2 = g2.to(x_.scalar_type());
  if (relu_here_) g2 = api::binary(g2.contiguous(), y_, BIN_RELU_BWD);
  const bool acc = weight_->take_accumulate();
  api::gemm(x_.t(), g2, c10::nullopt, ACT_NONE, 1.0, acc ? 1.0 : 0.0, weight_->grad);
  if (bias_) api::colsum(g2, 1.0, bias_->grad, bias_->take_accumulate());
  at::Tensor dx;
  if (need_input_grad) {
    dx = api::gemm(g2, weight_->master.t(), c10::nullopt, ACT_NONE, 1.0, 0.0, c10::nullopt,
                   mask_input_ ? c10::optional<at::Tensor>(x_) : c10::nullopt)
             .reshape(in_shape_);
  }
  return Tensor(dx, grad_output.device());
}

// ---------------------------------------------------------------- Activation
std::string ActivationLayer::type_name() const { return "Activation"; }

namespace {
const char* act_name(ActivationType t) {
  switch (t) {
    case ActivationType::ReLU: return "relu";
    case ActivationType::Sigmoid: return "sigmoid";
    case ActivationType::Tanh: return "tanh";
    case ActivationType::Softmax: return "softmax";
  }
  return "relu";
}
}  // namespace

std::string ActivationLayer::config_json() const {
  return std::string("{\"activation\":\"") + act_name(type_) + "\",\"type\":\"Activation\"}";
}

std::unique_ptr<ModernLayer> ActivationLayer::clone() const { return std::make_unique<ActivationLayer>(*this); }

Tensor ActivationLayer::forward(const Tensor& input) {
  at::Tensor y;
  switch (type_) {
    case ActivationType::ReLU: y = api::unary(input.data(), UN_RELU); break;
    case ActivationType::Sigmoid: y = api::unary(input.data(), UN_SIGMOID); break;
    case ActivationType::Tanh: y = api::unary(input.data(), UN_TANH); break;
    case ActivationType::Softmax: y = api::softmax(input.data()); break;
  }
  if (training_) saved_ = y;
  return Tensor(y, input.device());
}

Tensor ActivationLayer::backward(const Tensor& grad_output) {
  TORCH_CHECK(saved_.defined(), "dlvk: activation backward needs a training-mode forward");
  const at::Tensor g = grad_output.data().contiguous();
  at::Tensor dx;
  switch (type_) {
    case ActivationType::ReLU: dx = api::binary(g, saved_, BIN_RELU_BWD); break;
    case ActivationType::Sigmoid: dx = api::binary(g, saved_, BIN_SIGMOID_BWD); break;
    case ActivationType::Tanh: dx = api::binary(g, saved_, BIN_TANH_BWD); break;
    case ActivationType::Softmax: dx = api::softmax_bwd(saved_, g); break;
  }
  return Tensor(dx, grad_output.device());
}

// ---------------------------------------------------------------- Conv2D
Conv2DLayer::Conv2DLayer(size_t cin, size_t cout, size_t k, size_t s, size_t p, at::Generator& gen)
    : in_channels(cin), out_channels(cout), kernel_size(k), stride(s), padding(p) {
  const double k2 = (double)(k * k);
  const double std = std::sqrt(2.0 / ((double)cin * k2 + (double)cout * k2));
  weight_ = &add_param("weight", at::randn({(int64_t)cout, (int64_t)cin, (int64_t)k, (int64_t)k}, gen) * std);
  bias_ = &add_param("bias", at::zeros({(int64_t)cout}));
}

std::unique_ptr<ModernLayer> Conv2DLayer::clone() const {
  auto c = std::make_unique<Conv2DLayer>(*this);
  c->weight_ = c->params_[0].get();
  c->bias_ = c->params_[1].get();
  return c;
}

std::string Conv2DLayer::config_json() const {
  return "{\"activation\":null,\"in_channels\":" + std::to_string(in_channels) +
         ",\"kernel_size\":" + std::to_string(kernel_size) + ",\"out_channels\":" + std::to_string(out_channels) +
         ",\"padding\":" + std::to_string(padding) + ",\"stride\":" + std::to_string(stride) +
         ",\"type\":\"Conv2D\",\"use_bias\":true}";
}

Tensor Conv2DLayer::forward(const Tensor& input) { return forward_fused(input, false); }

Tensor Conv2DLayer::forward_fused(const Tensor& input, bool relu) {
  at::Tensor x = input.data().contiguous();
  at::Tensor y = api::conv2d_fwd(x, weight_->master, bias_->master, (int)stride, (int)padding, relu);
  relu_ = relu;
  if (training_) {
    x_ = x;
    y_ = relu ? y : at::Tensor();
  }
  return Tensor(y, input.device());
}

Tensor Conv2DLayer::backward(const Tensor& grad_output) {
  TORCH_CHECK(x_.defined(), "dlvk: Conv2D backward needs a training-mode forward");
  at::Tensor g = grad_output.data().contiguous();
  if (g.scalar_type() != x_.scalar_type()) g = g.to(x_.scalar_type());
  if (relu_) g = api::binary(g, y_, BIN_RELU_BWD);
  const bool acc = weight_->take_accumulate();
  bias_->take_accumulate();
  api::conv2d_wgrad(x_, g, weight_->grad, bias_->grad, (int)stride, (int)padding, acc);
  at::Tensor dx;
  if (need_input_grad) dx = api::conv2d_dgrad(g, weight_->master, sizes_of(x_), (int)stride, (int)padding, c10::nullopt);
  return Tensor(dx, grad_output.device());
}

// ---------------------------------------------------------------- pooling
std::unique_ptr<ModernLayer> MaxPool2DLayer::clone() const { return std::make_unique<MaxPool2DLayer>(*this); }
std::string MaxPool2DLayer::config_json() const {
  return "{\"pool_size\":" + std::to_string(pool_size) + ",\"stride\":" + std::to_string(stride) +
         ",\"type\":\"MaxPool2D\"}";
}
Tensor MaxPool2DLayer::forward(const Tensor& input) {
  at::Tensor x = input.data().contiguous();
  H_ = x.size(2);
  W_ = x.size(3);
  auto r = api::maxpool_fwd(x, (int)pool_size, (int)stride);
  if (training_) idx_ = r.second;
  return Tensor(r.first, input.device());
}
Tensor MaxPool2DLayer::backward(const Tensor& g) {
  TORCH_CHECK(idx_.defined(), "dlvk: MaxPool2D backward needs a training-mode forward");
  return Tensor(api::maxpool_bwd(g.data().contiguous(), idx_, (int)H_, (int)W_, (int)pool_size, (int)stride),
                g.device());
}

std::unique_ptr<ModernLayer> AvgPool2DLayer::clone() const { return std::make_unique<AvgPool2DLayer>(*this); }
std::string AvgPool2DLayer::config_json() const {
  return "{\"pool_size\":" + std::to_string(pool_size) + ",\"stride\":" + std::to_string(stride) +
         ",\"type\":\"AvgPool2D\"}";
}
Tensor AvgPool2DLayer::forward(const Tensor& input) {
  at::Tensor x = input.data().contiguous();
  H_ = x.size(2);
  W_ = x.size(3);
  return Tensor(api::avgpool_fwd(x, (int)pool_size, (int)stride), input.device());
}
Tensor AvgPool2DLayer::backward(const Tensor& g) {
  return Tensor(api::avgpool_bwd(g.data().contiguous(), (int)H_, (int)W_, (int)pool_size, (int)stride), g.device());
}

// ---------------------------------------------------------------- BatchNorm
BatchNormLayer::BatchNormLayer(size_t n, bool two_d, double momentum, double eps)
    : num_features(n), momentum(momentum), eps(eps), two_d_(two_d) {
  gamma_ = &add_param("gamma", at::ones({(int64_t)n}));
  beta_ = &add_param("beta", at::zeros({(int64_t)n}));
  running_mean = at::zeros({(int64_t)n});
  running_var = at::ones({(int64_t)n});
}

std::unique_ptr<ModernLayer> BatchNormLayer::clone() const {
  auto c = std::make_unique<BatchNormLayer>(*this);
  c->gamma_ = c->params_[0].get();
  c->beta_ = c->params_[1].get();
  c->running_mean = running_mean.clone();
  c->running_var = running_var.clone();
  return c;
}

std::string BatchNormLayer::config_json() const {
  return "{\"eps\":" + json::num(eps) + ",\"momentum\":" + json::num(momentum) +
         ",\"num_features\":" + std::to_string(num_features) + ",\"type\":" + json::str(type_name()) + "}";
}

std::vector<std::pair<std::string, at::Tensor*>> BatchNormLayer::buffers() {
  return {{"running_mean", &running_mean}, {"running_var", &running_var}};
}

Tensor BatchNormLayer::forward(const Tensor& input) {
  at::Tensor x = input.data().contiguous();
  if (running_mean.device() != x.device()) {
    running_mean = running_mean.to(x.device());
    running_var = running_var.to(x.device());
  }
  auto r = api::batchnorm_fwd(x, gamma_->master, beta_->master, running_mean, running_var, momentum, eps, training_);
  if (training_) {
    x_ = x;
    mean_ = r[1];
    rstd_ = r[2];
  }
  return Tensor(r[0], input.device());
}

Tensor BatchNormLayer::backward(const Tensor& g) {
  TORCH_CHECK(x_.defined(), "dlvk: BatchNorm backward needs a training-mode forward");
  const bool acc = gamma_->take_accumulate();
  beta_->take_accumulate();
  at::Tensor dx = api::batchnorm_bwd(x_, g.data().contiguous().to(x_.scalar_type()), mean_, rstd_, gamma_->master,
                                     beta_->master, gamma_->grad, beta_->grad, acc);
  return Tensor(dx, g.device());
}

// ---------------------------------------------------------------- Dropout / Flatten
std::unique_ptr<ModernLayer> DropoutLayer::clone() const { return std::make_unique<DropoutLayer>(*this); }
std::string DropoutLayer::config_json() const {
  return "{\"rate\":" + json::num((double)rate) + ",\"type\":\"Dropout\"}";
}
Tensor DropoutLayer::forward(const Tensor& input) {
  if (!training_ || rate <= 0.f) return input;
  used_step_ = *step_;
  return Tensor(api::dropout(input.data().contiguous(), rate, site_, *seed_, used_step_), input.device());
}
Tensor DropoutLayer::backward(const Tensor& g) {
  if (!training_ || rate <= 0.f) return g;
  return Tensor(api::dropout(g.data().contiguous(), rate, site_, *seed_, used_step_), g.device());
}

Tensor FlattenLayer::forward(const Tensor& input) {
  in_shape_ = sizes_of(input.data());
  return Tensor(input.data().reshape({input.data().size(0), -1}), input.device());
}
Tensor FlattenLayer::backward(const Tensor& g) { return Tensor(g.data().reshape(in_shape_), g.device()); }

// ---------------------------------------------------------------- accessors
std::vector<size_t> window_output_shape(const std::vector<size_t>& input_shape, size_t channels, size_t k,
                                        size_t stride, size_t padding) {
  const size_t r = input_shape.size();
  if (r != 3 && r != 4) throw std::invalid_argument("window_output_shape: expected an NCHW or CHW shape");
  if (stride == 0) throw std::invalid_argument("window_output_shape: stride 0");
  std::vector<size_t> out = input_shape;
  for (size_t d = r - 2; d < r; ++d) {
    const size_t padded = input_shape[d] + 2 * padding;
    if (padded < k) throw std::invalid_argument("window_output_shape: window larger than the padded input");
    out[d] = (padded - k) / stride + 1;
  }
  if (channels) out[r - 3] = channels;
  return out;
}

void BatchNormLayer::copy_into(at::Tensor& dst, const Tensor& src, const char* what) {
  if (!src.defined() || src.data().numel() != dst.numel())
    throw std::invalid_argument(std::string("BatchNorm ") + what + ": element count does not match");
  dst.copy_(src.data().reshape(dst.sizes()));
}

void DropoutLayer::set_dropout_rate(float r) {
  if (!(r >= 0.f && r < 1.f)) throw std::invalid_argument("dropout rate must be in [0, 1)");
  rate = r;
}

}  // namespace dlvk
