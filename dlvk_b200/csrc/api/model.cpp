// C++ API: Sequential and ModelTrainer (include/dlvk/model/model.h:15-143,
// src/model/model.cpp:20-318 of the reference).  Execution restates the
// Python package's Sequential (dlvk_b200/models/sequential.py): the same
// fusion plan, flat parameter layout, step counter and `.dlvk` metadata.
#include "dlvk/model/model.h"

#include <ATen/CPUGeneratorImpl.h>

#include <algorithm>
#include <cstdio>
#include <iostream>
#include <cstring>
#include <sstream>

#include "dispatch.h"
#include "dlvk/common.h"
#include "dlvk/io.h"
#include "json_util.h"

namespace dlvk {

namespace {
constexpr int64_t kAlignElems = 64;  // 256 bytes of fp32 per parameter slot
int64_t round_up(int64_t n, int64_t a) { return (n + a - 1) / a * a; }

io::TensorRecord record_of(const std::string& name, const at::Tensor& t) {
  at::Tensor c = t.detach().contiguous().to(c10::kCPU);
  io::TensorRecord r;
  r.name = name;
  switch (c.scalar_type()) {
    case at::kFloat: r.dtype = (uint32_t)DType::F32; break;
    case at::kBFloat16: r.dtype = (uint32_t)DType::BF16; break;
    case at::kInt: r.dtype = (uint32_t)DType::I32; break;
    case at::kLong: r.dtype = (uint32_t)DType::I64; break;
    default: TORCH_CHECK(false, "dlvk: cannot save dtype ", c.scalar_type());
  }
  for (auto d : c.sizes()) r.dims.push_back((uint64_t)d);
  r.data.assign(reinterpret_cast<const char*>(c.data_ptr()), (size_t)(c.numel() * c.element_size()));
  return r;
}
}  // namespace

Sequential::Sequential(std::shared_ptr<CudaDevice> device, uint64_t seed)
    : device_(device ? std::move(device) : CudaDevice::cpu()),
      gen_(at::detail::createCPUGenerator(seed)),
      seed_(seed) {
  if (!device_->is_initialized()) device_->initialize();
}

Sequential::~Sequential() = default;

void Sequential::add(std::unique_ptr<ModernLayer> layer) {
  TORCH_CHECK(!built_, "dlvk: cannot add layers after the model was built");
  layers_.push_back(std::move(layer));
  plan_.clear();
}

std::unique_ptr<Sequential> Sequential::clone() const {
  auto c = std::make_unique<Sequential>(device_, seed_);
  for (const auto& l : layers_) {
    if (const auto* d = dynamic_cast<const DropoutLayer*>(l.get()))
      c->add(std::make_unique<DropoutLayer>(d->rate, ++c->dropout_sites_, &c->seed_, &c->step_));
    else
      c->add(l->clone());
  }
  c->step_ = step_;
  c->set_training(training_);
  return c;
}

void Sequential::add_dense(size_t in, size_t out, bool use_bias) {
  add(std::make_unique<DenseLayer>(in, out, use_bias, gen_));
}
void Sequential::add_conv2d(size_t cin, size_t cout, size_t k, size_t s, size_t p) {
  add(std::make_unique<Conv2DLayer>(cin, cout, k, s, p, gen_));
}
void Sequential::add_maxpool2d(size_t k, size_t s) { add(std::make_unique<MaxPool2DLayer>(k, s)); }
void Sequential::add_avgpool2d(size_t k, size_t s) { add(std::make_unique<AvgPool2DLayer>(k, s)); }
void Sequential::add_batchnorm1d(size_t n) { add(std::make_unique<BatchNormLayer>(n, false)); }
void Sequential::add_batchnorm2d(size_t n) { add(std::make_unique<BatchNormLayer>(n, true)); }
void Sequential::add_dropout(float rate) {
  add(std::make_unique<DropoutLayer>(rate, ++dropout_sites_, &seed_, &step_));
}
void Sequential::add_relu() { add(std::make_unique<ActivationLayer>(ActivationType::ReLU)); }
void Sequential::add_sigmoid() { add(std::make_unique<ActivationLayer>(ActivationType::Sigmoid)); }
void Sequential::add_tanh() { add(std::make_unique<ActivationLayer>(ActivationType::Tanh)); }
void Sequential::add_softmax() { add(std::make_unique<ActivationLayer>(ActivationType::Softmax)); }
void Sequential::add_flatten() { add(std::make_unique<FlattenLayer>()); }

std::vector<Parameter*> Sequential::parameters() {
  std::vector<Parameter*> out;
  for (auto& l : layers_)
    for (Parameter* p : l->parameters()) out.push_back(p);
  return out;
}

// Packs every parameter into flat fp32 buffers on the model's device, in
// reverse registration order (gradients become ready last layer first).
void Sequential::build() {
  if (built_) return;
  auto params = parameters();
  std::vector<Parameter*> order(params.rbegin(), params.rend());
  int64_t off = 0;
  for (Parameter* p : order) {
    p->offset = off;
    off += round_up(p->numel(), kAlignElems);
  }
  numel_ = std::max<int64_t>(off, kAlignElems);
  auto opts = at::TensorOptions().dtype(at::kFloat).device(device_->device());
  master_ = at::zeros({numel_}, opts);
  grad_ = at::zeros({numel_}, opts);
  for (Parameter* p : order) {
    master_.narrow(0, p->offset, p->numel()).copy_(p->master.to(device_->device(), at::kFloat).reshape({-1}));
    p->master = master_.narrow(0, p->offset, p->numel()).view(p->shape);
    p->grad = grad_.narrow(0, p->offset, p->numel()).view(p->shape);
    p->store = this;
  }
  for (auto& l : layers_)
    if (auto* bn = dynamic_cast<BatchNormLayer*>(l.get())) {
      bn->running_mean = bn->running_mean.to(device_->device());
      bn->running_var = bn->running_var.to(device_->device());
    }
  if (!layers_.empty()) layers_[0]->need_input_grad = false;
  built_ = true;
}

bool Sequential::has_trailing_softmax() const {
  if (layers_.empty()) return false;
  auto* a = dynamic_cast<const ActivationLayer*>(layers_.back().get());
  return a && a->activation() == ActivationType::Softmax;
}

// Groups layers into fused steps, as the Python package's Sequential does:
// Dense + ReLU (GEMM epilogue; a following Dense applies the ReLU backward in
// its dX GEMM) and Conv2D + ReLU.
void Sequential::make_plan() {
  plan_.clear();
  bool relu_feeds_dense = false;
  size_t i = 0;
  auto is_relu = [&](size_t j) {
    if (j >= layers_.size()) return false;
    auto* a = dynamic_cast<ActivationLayer*>(layers_[j].get());
    return a && a->activation() == ActivationType::ReLU;
  };
  while (i < layers_.size()) {
    ModernLayer* cur = layers_[i].get();
    auto* dense = dynamic_cast<DenseLayer*>(cur);
    auto* conv = dynamic_cast<Conv2DLayer*>(cur);
    if (dense && is_relu(i + 1)) {
      const bool feeds = i + 2 < layers_.size() && dynamic_cast<DenseLayer*>(layers_[i + 2].get()) != nullptr;
      const bool mask_in = relu_feeds_dense;
      plan_.push_back({i, 2, [dense, feeds, mask_in](const Tensor& x) {
                         return dense->forward_fused(x, ACT_RELU, mask_in, feeds);
                       }});
      relu_feeds_dense = feeds;
      i += 2;
      continue;
    }
    if (dense && relu_feeds_dense) {
      plan_.push_back({i, 1, [dense](const Tensor& x) { return dense->forward_fused(x, ACT_NONE, true, false); }});
      relu_feeds_dense = false;
      i += 1;
      continue;
    }
    relu_feeds_dense = false;
    if (conv && is_relu(i + 1)) {
      plan_.push_back({i, 2, [conv](const Tensor& x) { return conv->forward_fused(x, true); }});
      i += 2;
      continue;
    }
    plan_.push_back({i, 1, [cur](const Tensor& x) { return cur->forward(x); }});
    i += 1;
  }
}

at::Tensor Sequential::prepare_input(const Tensor& x) const {
  at::Tensor t = x.data();
  if (t.device() != device_->device()) t = t.to(device_->device());
  if (t.is_floating_point() && t.scalar_type() != at::kFloat) t = api::unary(t, UN_COPY).to(at::kFloat);
  return t;
}

Tensor Sequential::run(const Tensor& x, size_t upto) {
  build();
  if (plan_.empty()) make_plan();
  Tensor cur = x;
  size_t consumed = 0, steps = 0;
  for (auto& st : plan_) {
    if (consumed + st.count > upto) break;
    cur = st.fwd(cur);
    for (size_t j = st.first; j < st.first + st.count; ++j)
      layers_[j]->output_shape = std::vector<int64_t>(cur.data().sizes().begin(), cur.data().sizes().end());
    consumed += st.count;
    ++steps;
  }
  last_out_ = cur;
  last_steps_ = steps;
  return cur;
}

Tensor Sequential::forward(const Tensor& input) {
  return run(Tensor(prepare_input(input), device_), layers_.size());
}

Tensor Sequential::forward_logits(const Tensor& input) {
  const size_t n = layers_.size() - (has_trailing_softmax() ? 1 : 0);
  return run(Tensor(prepare_input(input), device_), n);
}

void Sequential::backward(const Tensor& grad_output) {
  TORCH_CHECK(training_ && last_out_.defined(), "dlvk: backward() needs a preceding forward() in training mode");
  Tensor g(grad_output.data().to(last_out_.data().device(), last_out_.data().scalar_type()), device_);
  for (size_t i = last_steps_; i-- > 0;) g = layers_[plan_[i].first]->backward(g);
  // Parameters that received no gradient this step get zeros.
  for (Parameter* p : parameters())
    if (p->fresh) {
      p->grad.zero_();
      p->fresh = false;
    }
}

void Sequential::zero_grad() {
  build();
  for (Parameter* p : parameters()) p->fresh = true;
}

void Sequential::update_parameters(Optimizer& optimizer) { optimizer.step(*this); }

void Sequential::set_training(bool training) {
  training_ = training;
  for (auto& l : layers_) l->set_training(training);
}

Tensor Sequential::train_step(const Tensor& x, const Tensor& y, LossFunction& loss, Optimizer& optimizer) {
  build();
  zero_grad();
  ++step_;
  auto* ce = dynamic_cast<CrossEntropyLoss*>(&loss);
  const bool fused = ce != nullptr && has_trailing_softmax();
  Tensor out = fused ? forward_logits(x) : forward(x);
  std::pair<Tensor, Tensor> lg = fused ? ce->value_and_grad_from_logits(out, y) : loss.value_and_grad(out, y);
  backward(lg.second);
  optimizer.step(*this);
  return lg.first;
}

std::string Sequential::summary() const {
  std::ostringstream o;
  auto pad = [](std::string s, size_t w, bool right) {
    if (s.size() >= w) return s;
    return right ? std::string(w - s.size(), ' ') + s : s + std::string(w - s.size(), ' ');
  };
  o << "Model: Sequential\n" << std::string(60, '-') << "\n"
    << pad("Layer (type)", 24, false) << pad("Output Shape", 24, false) << pad("Param #", 12, true) << "\n"
    << std::string(60, '=') << "\n";
  for (const auto& l : layers_) {
    LayerInfo info = l->get_layer_info();
    if (auto* a = dynamic_cast<const ActivationLayer*>(l.get())) {
      static const char* names[] = {"ReLU", "Sigmoid", "Tanh", "Softmax"};
      info.type = names[(int)a->activation()];
    }
    o << pad(info.type, 24, false) << pad(info.output_shape_str, 24, false)
      << pad(std::to_string(info.parameter_count), 12, true) << "\n";
  }
  o << std::string(60, '=') << "\n" << "Total params: " << parameter_count();
  return o.str();
}

size_t Sequential::parameter_count() const {
  size_t n = 0;
  for (const auto& l : layers_) n += l->parameter_count();
  return n;
}

std::vector<std::pair<std::string, at::Tensor*>> Sequential::state_tensors() const {
  std::vector<std::pair<std::string, at::Tensor*>> out;
  for (size_t i = 0; i < layers_.size(); ++i)
    for (auto& kv : layers_[i]->state_tensors()) out.emplace_back("layers." + std::to_string(i) + "." + kv.first, kv.second);
  return out;
}

std::string Sequential::architecture_json() const {
  std::string s = "[";
  for (size_t i = 0; i < layers_.size(); ++i) s += (i ? "," : "") + layers_[i]->config_json();
  return s + "]";
}

std::string Sequential::meta_json(const Optimizer* optimizer) const {
  std::string s = "{\"architecture\":" + architecture_json() + ",\"compute_dtype\":\"float32\"" +
                  ",\"format_version\":2,\"framework\":\"dlvk_b200\"";
  if (optimizer != nullptr) s += ",\"optimizer\":" + optimizer->state_meta_json(*this);
  s += ",\"rng\":{\"seed\":" + std::to_string(seed_) + ",\"step\":" + std::to_string(step_) + "}}";
  return s;
}

void Sequential::save_weights(const std::string& filepath) const { save_weights(filepath, nullptr); }
void Sequential::load_weights(const std::string& filepath) { load_weights(filepath, nullptr); }

void Sequential::save_weights(const std::string& filepath, const Optimizer* optimizer) const {
  const_cast<Sequential*>(this)->build();
  std::vector<io::TensorRecord> recs;
  for (auto& kv : state_tensors()) recs.push_back(record_of(kv.first, *kv.second));
  if (optimizer != nullptr)
    for (auto& kv : const_cast<Optimizer*>(optimizer)->state_tensors(*this)) recs.push_back(record_of(kv.first, *kv.second));
  io::save_v2(filepath, meta_json(optimizer), recs);
}

namespace {
// The integer value of "key": in a flat JSON object (the `.dlvk` rng block).
int64_t json_int(const std::string& js, const std::string& key, int64_t dflt) {
  const size_t k = js.find("\"" + key + "\":");
  if (k == std::string::npos) return dflt;
  return std::stoll(js.substr(k + key.size() + 3));
}
}  // namespace

void Sequential::load_weights(const std::string& filepath, Optimizer* optimizer) {
  build();
  io::DlvkFile f = io::load(filepath);
  TORCH_CHECK(f.variant == "v2", "dlvk: load_weights reads .dlvk v2 files (got ", f.variant, ")");
  auto find = [&](const std::string& name) -> const io::TensorRecord* {
    for (const auto& r : f.tensors)
      if (r.name == name) return &r;
    return nullptr;
  };
  auto restore = [&](const std::string& name, at::Tensor* t) {
    const io::TensorRecord* r = find(name);
    TORCH_CHECK(r != nullptr, "dlvk: .dlvk file has no tensor '", name, "'");
    TORCH_CHECK(r->data.size() == (size_t)(t->numel() * t->element_size()), "dlvk: ", name, ": size mismatch");
    at::Tensor host = at::empty(t->sizes(), t->options().device(c10::kCPU));
    std::memcpy(host.data_ptr(), r->data.data(), r->data.size());
    t->copy_(host);
  };
  for (auto& kv : state_tensors()) restore(kv.first, kv.second);
  const size_t rng = f.meta_json.find("\"rng\":");
  if (rng != std::string::npos) {
    const std::string blk = f.meta_json.substr(rng, f.meta_json.find('}', rng) - rng);
    seed_ = (uint64_t)json_int(blk, "seed", (int64_t)seed_);
    step_ = json_int(blk, "step", 0);
  }
  const size_t ob = f.meta_json.find("\"optimizer\":");
  if (optimizer != nullptr && ob != std::string::npos) {
    for (auto& kv : optimizer->state_tensors(*this))
      if (find(kv.first) != nullptr) restore(kv.first, kv.second);
    const std::string blk = f.meta_json.substr(ob, f.meta_json.find('}', ob) - ob);
    double lr = optimizer->get_learning_rate();
    const size_t k = blk.find("\"lr\":");
    if (k != std::string::npos) lr = std::stod(blk.substr(k + 5));
    optimizer->load_state_meta(*this, json_int(blk, "step", 0), lr);
  }
}

// ---------------------------------------------------------------- ModelTrainer
ModelTrainer::ModelTrainer(Sequential* model) : model_(model) {}

void ModelTrainer::compile(std::unique_ptr<Optimizer> optimizer, std::unique_ptr<LossFunction> loss_function) {
  optimizer_ = std::move(optimizer);
  loss_ = std::move(loss_function);
}

void ModelTrainer::add_callback(std::unique_ptr<TrainingCallback> cb) { callbacks_.push_back(std::move(cb)); }

std::pair<float, float> ModelTrainer::batch_metrics(const Tensor& x, const Tensor& y) {
  Tensor out = model_->forward(x);
  at::Tensor o = out.data().to(c10::kCPU, at::kFloat);
  at::Tensor t = y.data().to(c10::kCPU);
  at::Tensor o2 = o.reshape({-1, o.size(-1)});
  at::Tensor lab = t.is_floating_point() ? t.reshape({o2.size(0), -1}).argmax(-1) : t.reshape({-1}).to(at::kLong);
  const float acc = (float)(o2.argmax(-1) == lab).to(at::kFloat).mean().item<float>();
  float loss;
  if (model_->has_trailing_softmax() && dynamic_cast<CrossEntropyLoss*>(loss_.get())) {
    at::Tensor p = o2.clamp_min(1e-8);
    loss = -(at::log(p).gather(1, lab.unsqueeze(1))).mean().item<float>();
  } else {
    loss = loss_->forward(std::make_shared<Tensor>(out), std::make_shared<Tensor>(y))->data().item<float>();
  }
  return {loss, acc};
}

std::vector<TrainingMetrics> ModelTrainer::fit(const Tensor& x_train, const Tensor& y_train, size_t epochs,
                                               size_t batch_size, float validation_split, bool verbose) {
  TORCH_CHECK(optimizer_ && loss_, "dlvk: ModelTrainer::fit before compile()");
  const int64_t n = x_train.data().size(0);
  const int64_t n_val = (int64_t)((double)n * validation_split);
  const int64_t n_tr = n - n_val;
  std::vector<TrainingMetrics> history;
  for (auto& cb : callbacks_) cb->on_train_begin();
  for (size_t ep = 0; ep < epochs; ++ep) {
    for (auto& cb : callbacks_) cb->on_epoch_begin(ep);
    model_->set_training(true);
    double loss_sum = 0.0;
    size_t batches = 0;
    for (int64_t s = 0; s < n_tr; s += (int64_t)batch_size, ++batches) {
      const int64_t e = std::min<int64_t>(n_tr, s + (int64_t)batch_size);
      for (auto& cb : callbacks_) cb->on_batch_begin(batches);
      Tensor xb(x_train.data().slice(0, s, e), x_train.device());
      Tensor yb(y_train.data().slice(0, s, e), y_train.device());
      const float l = model_->train_step(xb, yb, *loss_, *optimizer_).data().item<float>();
      loss_sum += l;
      TrainingMetrics bm;
      bm.loss = l;
      bm.epoch = ep;
      bm.batch = batches;
      for (auto& cb : callbacks_) cb->on_batch_end(batches, bm);
    }
    TrainingMetrics m;
    m.epoch = ep;
    m.batch = batches;
    m.loss = batches ? (float)(loss_sum / (double)batches) : 0.f;
    model_->set_training(false);
    m.accuracy = batch_metrics(Tensor(x_train.data().slice(0, 0, n_tr), x_train.device()),
                               Tensor(y_train.data().slice(0, 0, n_tr), y_train.device())).second;
    if (n_val > 0) {
      auto vm = batch_metrics(Tensor(x_train.data().slice(0, n_tr, n), x_train.device()),
                              Tensor(y_train.data().slice(0, n_tr, n), y_train.device()));
      m.validation_loss = vm.first;
      m.validation_accuracy = vm.second;
    }
    model_->set_training(true);
    if (verbose)
      std::printf("epoch %zu: loss %.4f acc %.4f val_loss %.4f val_acc %.4f\n", ep + 1, m.loss, m.accuracy,
                  m.validation_loss, m.validation_accuracy);
    history.push_back(m);
    for (auto& cb : callbacks_) cb->on_epoch_end(ep, m);
  }
  for (auto& cb : callbacks_) cb->on_train_end();
  return history;
}

TrainingMetrics ModelTrainer::evaluate(const Tensor& x, const Tensor& y, size_t batch_size) {
  model_->set_training(false);
  const int64_t n = x.data().size(0);
  double loss = 0.0, acc = 0.0;
  for (int64_t s = 0; s < n; s += (int64_t)batch_size) {
    const int64_t e = std::min<int64_t>(n, s + (int64_t)batch_size);
    auto bm = batch_metrics(Tensor(x.data().slice(0, s, e), x.device()), Tensor(y.data().slice(0, s, e), y.device()));
    loss += bm.first * (double)(e - s);
    acc += bm.second * (double)(e - s);
  }
  model_->set_training(true);
  TrainingMetrics m;
  m.loss = n ? (float)(loss / (double)n) : 0.f;
  m.accuracy = n ? (float)(acc / (double)n) : 0.f;
  return m;
}

Tensor ModelTrainer::predict(const Tensor& x, size_t batch_size) {
  model_->set_training(false);
  std::vector<at::Tensor> outs;
  const int64_t n = x.data().size(0);
  for (int64_t s = 0; s < n; s += (int64_t)batch_size)
    outs.push_back(model_->forward(Tensor(x.data().slice(0, s, std::min<int64_t>(n, s + (int64_t)batch_size)), x.device())).data());
  model_->set_training(true);
  return Tensor(at::cat(outs, 0), model_->device());
}

}  // namespace dlvk
