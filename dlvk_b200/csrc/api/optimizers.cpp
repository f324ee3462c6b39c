// C++ API: optimizers over a model's flat parameter buffers.  The update
// sequence (advance the step, then one update over the whole buffer)
// restates the Python package's Optimizer.step (dlvk_b200/optim.py); on CUDA
// it uses the same device hyper-parameter block and optim.cu kernels.
#include "dlvk/optimizers/optimizers.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "dispatch.h"
#include "dlvk/aten_ops.h"
#include "dlvk/kernels.h"
#include "dlvk/model/model.h"
#include "json_util.h"

namespace dlvk {

struct Optimizer::State {
  Sequential* model = nullptr;
  at::Tensor m, v;        // flat fp32, parallel to the model's buffers
  at::Tensor hyper;       // device OptimHyper block (CUDA)
  at::Tensor clip;        // clip coefficient (1); the CUDA update reads it through the hyper block
  at::Tensor sumsq, scratch;  // norm-clipping work buffers (CUDA)
  bool clip_set = false;      // clip holds a norm-clipping coefficient
  int64_t step = 0;       // host step count
};

Optimizer::Optimizer(int kind, double lr, double beta1, double beta2, double eps, double momentum, double alpha,
                     double weight_decay)
    : kind_(kind), lr_(lr), beta1_(beta1), beta2_(beta2), eps_(eps), momentum_(momentum), alpha_(alpha),
      weight_decay_(weight_decay) {}

Optimizer::~Optimizer() = default;

SGD::SGD(double lr, double momentum, double wd) : Optimizer(OPT_SGD, lr, 0.9, 0.999, 1e-8, momentum, 0.99, wd) {}
Adam::Adam(double lr, double b1, double b2, double eps, double wd)
    : Optimizer(OPT_ADAM, lr, b1, b2, eps, 0.0, 0.99, wd) {}
RMSprop::RMSprop(double lr, double alpha, double eps) : Optimizer(OPT_RMSPROP, lr, 0.9, 0.999, eps, 0.0, alpha, 0.0) {}

namespace {
OptimHyper pack(double lr, double b1, double b2, double eps, double wd, double mom, double alpha, bool bc,
                const float* clip) {
  OptimHyper h;
  std::memset(&h, 0, sizeof h);
  h.lr = (float)lr;
  h.beta1 = (float)b1;
  h.beta2 = (float)b2;
  h.eps = (float)eps;
  h.weight_decay = (float)wd;
  h.momentum = (float)mom;
  h.alpha = (float)alpha;
  h.grad_scale = 1.f;
  h.bc1 = h.bc2 = 1.f;
  h.step = 0;
  h.bias_correction = bc ? 1 : 0;
  h.decoupled_wd = 0;
  h.clip_coef_ptr = clip;
  h.skip_flag_ptr = nullptr;
  return h;
}
}  // namespace

Optimizer::State& Optimizer::state(const Sequential& model) {
  auto it = states_.find(&model);
  if (it != states_.end()) return *it->second;
  auto st = std::make_unique<State>();
  auto& mdl = const_cast<Sequential&>(model);
  st->model = &mdl;
  const int64_t n = mdl.flat_numel();
  auto opts = mdl.master().options();
  if (kind_ == OPT_ADAM || kind_ == OPT_SGD) st->m = at::zeros({n}, opts);
  if (kind_ == OPT_ADAM || kind_ == OPT_RMSPROP) st->v = at::zeros({n}, opts);
  st->clip = at::ones({1}, opts);
  if (mdl.master().is_cuda()) {
    OptimHyper h = pack(lr_, beta1_, beta2_, eps_, weight_decay_, momentum_, alpha_, bias_correction_,
                        st->clip.data_ptr<float>());
    at::Tensor host = at::empty({(int64_t)sizeof(OptimHyper)}, at::kByte);
    std::memcpy(host.data_ptr(), &h, sizeof h);
    st->hyper = host.to(mdl.master().device());
  }
  auto& ref = *st;
  states_[&model] = std::move(st);
  return ref;
}

const Optimizer::State* Optimizer::find_state(const Sequential& model) const {
  auto it = states_.find(&model);
  return it == states_.end() ? nullptr : it->second.get();
}

void Optimizer::set_learning_rate(double lr) {
  lr_ = lr;
  for (auto& kv : states_) {
    if (!kv.second->hyper.defined()) continue;
    const float f = (float)lr;
    at::Tensor b = at::empty({4}, at::kByte);
    std::memcpy(b.data_ptr(), &f, 4);
    kv.second->hyper.narrow(0, offsetof(OptimHyper, lr), 4).copy_(b);
  }
}

void Optimizer::set_grad_clip_norm(double max_norm) {
  TORCH_CHECK(max_norm > 0.0, "dlvk: set_grad_clip_norm needs max_norm > 0");
  clip_norm_ = max_norm;
  use_clip_norm_ = true;
}

void Optimizer::set_grad_clip_value(double min_val, double max_val) {
  TORCH_CHECK(min_val <= max_val, "dlvk: set_grad_clip_value: empty range");
  clip_min_ = min_val;
  clip_max_ = max_val;
  use_clip_value_ = true;
}

void Optimizer::disable_grad_clipping() { use_clip_norm_ = use_clip_value_ = false; }

// Value clamp, then the norm-clipping coefficient into st.clip: on CUDA by
// the grad_stats kernel (sum of squares and coefficient stay on the device),
// on CPU from the fp32 norm, as the Python package's Optimizer.prepare_grads.
void Optimizer::prepare_grads(State& st, at::Tensor& grad) {
  if (use_clip_value_) {
    if (grad.is_cuda())
      aten::unary_op(grad, UN_CLAMP, clip_min_, clip_max_, grad, c10::nullopt);
    else
      grad.clamp_(clip_min_, clip_max_);
  }
  if (!use_clip_norm_) {
    if (st.clip_set) st.clip.fill_(1.0);  // clipping was switched off since the last step
    st.clip_set = false;
    return;
  }
  st.clip_set = true;
  if (grad.is_cuda()) {
    if (!st.sumsq.defined()) {
      st.sumsq = at::zeros({1}, grad.options());
      st.scratch = at::empty({(int64_t)grad_stats_scratch_floats()}, grad.options());
    }
    aten::grad_stats_op(grad, 1.0, clip_norm_, st.sumsq, c10::nullopt, st.clip, false, st.scratch, c10::nullopt);
  } else {
    const double norm = grad.norm().item<double>();
    st.clip.fill_(std::min(1.0, clip_norm_ / (norm + 1e-6)));
  }
}

void Optimizer::advance(State& st) {
  st.step += 1;
  if (st.hyper.defined()) aten::optim_advance_op(st.hyper);
}

void Optimizer::update_range(State& st, at::Tensor& master, at::Tensor& grad, int64_t start, int64_t end) {
  at::Tensor p = master.narrow(0, start, end - start);
  at::Tensor g = grad.narrow(0, start, end - start);
  api::OptT m = st.m.defined() ? api::OptT(st.m.narrow(0, start, end - start)) : c10::nullopt;
  api::OptT v = st.v.defined() ? api::OptT(st.v.narrow(0, start, end - start)) : c10::nullopt;
  api::CpuHyper h{lr_, beta1_, beta2_, eps_, weight_decay_, momentum_, alpha_, bias_correction_, st.step};
  if (!st.hyper.defined() && use_clip_norm_) {
    // The CPU update has no clip pointer: scale a copy of the gradient.
    at::Tensor gs = g * st.clip.item<float>();
    api::optim_update(kind_, st.hyper, h, p, gs, m, v);
    return;
  }
  api::optim_update(kind_, st.hyper, h, p, g, m, v);
}

void Optimizer::step(Sequential& model) {
  model.build();
  State& st = state(model);
  advance(st);
  prepare_grads(st, model.grad());
  update_range(st, model.master(), model.grad(), 0, model.flat_numel());
}

void Optimizer::update(ModernLayer* layer) {
  auto params = layer->parameters();
  if (params.empty()) return;
  TORCH_CHECK(params[0]->store != nullptr, "dlvk: Optimizer::update needs a layer of a built Sequential");
  auto* model = static_cast<Sequential*>(const_cast<void*>(params[0]->store));
  State& st = state(*model);
  advance(st);
  prepare_grads(st, model->grad());
  for (Parameter* p : params) update_range(st, model->master(), model->grad(), p->offset, p->offset + p->numel());
}

int64_t Optimizer::step_count(const Sequential& model) const {
  const State* st = find_state(model);
  if (st == nullptr) return 0;
  if (st->hyper.defined()) {
    at::Tensor host = st->hyper.to(c10::kCPU);
    int step = 0;
    std::memcpy(&step, host.data_ptr<uint8_t>() + offsetof(OptimHyper, step), 4);
    return step;
  }
  return st->step;
}

void Optimizer::load_state_meta(const Sequential& model, int64_t step, double lr) {
  State& st = state(model);
  st.step = step;
  set_learning_rate(lr);
  if (!st.hyper.defined()) return;
  auto put = [&](size_t off, const void* v) {
    at::Tensor b = at::empty({4}, at::kByte);
    std::memcpy(b.data_ptr(), v, 4);
    st.hyper.narrow(0, (int64_t)off, 4).copy_(b);
  };
  const int s32 = (int)step;
  put(offsetof(OptimHyper, step), &s32);
  if (bias_correction_ && step > 0) {
    const float bc1 = (float)(1.0 / (1 - std::pow(beta1_, (double)step)));
    const float bc2 = (float)(1.0 / (1 - std::pow(beta2_, (double)step)));
    put(offsetof(OptimHyper, bc1), &bc1);
    put(offsetof(OptimHyper, bc2), &bc2);
  }
}

std::vector<std::pair<std::string, at::Tensor*>> Optimizer::state_tensors(const Sequential& model) {
  State& st = state(model);
  std::vector<std::pair<std::string, at::Tensor*>> out;
  if (st.m.defined()) out.emplace_back("optim.m", &st.m);
  if (st.v.defined()) out.emplace_back("optim.v", &st.v);
  return out;
}

std::string Optimizer::state_meta_json(const Sequential& model) const {
  return "{\"alpha\":" + json::num(alpha_) + ",\"beta1\":" + json::num(beta1_) + ",\"beta2\":" + json::num(beta2_) +
         ",\"bias_correction\":" + (bias_correction_ ? "true" : "false") + ",\"eps\":" + json::num(eps_) +
         ",\"lr\":" + json::num(lr_) + ",\"momentum\":" + json::num(momentum_) +
         ",\"step\":" + std::to_string(step_count(model)) + ",\"type\":" + json::str(name()) +
         ",\"weight_decay\":" + json::num(weight_decay_) + "}";
}

}  // namespace dlvk
