// C++ API program: the reference README's example model (README.md:60-78:
// Sequential Dense 784->128, ReLU, Dense 128->10, Softmax; batch-1 forward)
// and one training step of the 784-128-10 MLP on batch 32 (x ~ U[0, 1),
// labels uniform in [0, 10), generator seed 0; cross-entropy, Adam 1e-3).
//
//   cpp_api_mlp <cpu|cuda> <out_dir>
//
// Writes <out_dir>/loss.bin (fp32), grad.bin (the flat fp32 gradient
// buffer) and model.dlvk (weights + Adam state) for comparison with the
// Python API, and exercises Tensor / TensorOpsStatic / ModelTrainer.
#include <ATen/CPUGeneratorImpl.h>
#include <ATen/Parallel.h>

#include <cmath>
#include <cstdio>
#include <fstream>
#include <stdexcept>
#include <string>

#include "dlvk/dlvk.h"

namespace {
int fail(const std::string& what) {
  std::fprintf(stderr, "FAIL: %s\n", what.c_str());
  return 1;
}
void write_bytes(const std::string& path, const at::Tensor& t) {
  at::Tensor c = t.detach().contiguous().to(c10::kCPU);
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char*>(c.data_ptr()), (std::streamsize)(c.numel() * c.element_size()));
}
}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) return fail("usage: cpp_api_mlp <cpu|cuda> <out_dir>");
  const std::string mode = argv[1], out = argv[2];
  at::set_num_threads(1);
  auto device = mode == "cuda" ? std::make_shared<dlvk::CudaDevice>(0) : dlvk::CudaDevice::cpu();
  if (!device->initialize()) return fail("no CUDA device");
  std::printf("device %s (%s, %s, %llu bytes)\n", device->get_device_name().c_str(),
              device->get_device_type_string().c_str(), device->get_vulkan_version_string().c_str(),
              (unsigned long long)device->get_total_device_memory());
  if (device->is_cuda() && (device->get_max_workgroup_size() == 0 || device->get_total_device_memory() == 0))
    return fail("device getters");

  // README example: batch-1 forward of a freshly built model.
  {
    dlvk::Sequential model(device);
    model.add_dense(784, 128);
    model.add_relu();
    model.add_dense(128, 10);
    model.add_softmax();
    auto input = dlvk::Tensor::zeros(device, {1, 784});
    auto output = model.forward(input);
    if (output.shape() != std::vector<size_t>{1, 10}) return fail("README model output shape");
    auto s = output.sum()->to_vector();
    if (std::fabs(s[0] - 1.f) > 1e-5f) return fail("softmax output does not sum to 1");
    std::printf("%s\n", model.summary().c_str());
  }

  // Tensor / TensorOpsStatic basics.
  {
    auto a = dlvk::Tensor::from_vector(device, {2, 3}, {1, -2, 3, -4, 5, -6});
    auto b = dlvk::Tensor::from_vector(device, {3, 2}, {1, 0, 0, 1, 1, 1});
    auto c = a.matrix_multiply(b)->to_vector();  // [[4, 1], [-10, -1]]
    if (c != std::vector<float>({4, 1, -10, -1})) return fail("matrix_multiply");
    dlvk::Tensor r({2, 3}, dlvk::DataType::FLOAT32, device);
    if (!dlvk::TensorOpsStatic::relu(a, r) || r.to_vector() != std::vector<float>({1, 0, 3, 0, 5, 0}))
      return fail("TensorOpsStatic::relu");
    dlvk::Tensor bad({5}, dlvk::DataType::FLOAT32, device);
    if (dlvk::TensorOpsStatic::relu(a, bad)) return fail("TensorOpsStatic accepted a wrong result shape");
    if (a.sum(0)->to_vector() != std::vector<float>({-3, 3, -3})) return fail("sum(axis 0)");
    if (a.sum()->to_vector()[0] != -3.f) return fail("sum(all)");
    if (a.transpose()->shape() != std::vector<size_t>({3, 2})) return fail("transpose");
  }

  // The 784-128-10 MLP workload: one forward / backward / Adam step, batch 32.
  at::Generator g = at::detail::createCPUGenerator(0);
  at::Tensor x = at::rand({32, 784}, g);
  at::Tensor y = at::randint(0, 10, {32}, g);
  dlvk::Sequential model(device, 0);
  model.add_dense(784, 128);
  model.add_relu();
  model.add_dense(128, 10);
  model.add_softmax();
  dlvk::Adam adam(1e-3);
  dlvk::CrossEntropyLoss ce;
  dlvk::Tensor loss = model.train_step(dlvk::Tensor(x), dlvk::Tensor(y), ce, adam);
  write_bytes(out + "/loss.bin", loss.data().to(at::kFloat).reshape({1}));
  write_bytes(out + "/grad.bin", model.grad());
  model.save_weights(out + "/model.dlvk", &adam);
  std::printf("config1 loss %.6f\n", loss.data().item<float>());

  // Round trip: a fresh model loads the checkpoint and saves the same bytes.
  {
    dlvk::Sequential m2(device, 7);
    m2.add_dense(784, 128);
    m2.add_relu();
    m2.add_dense(128, 10);
    m2.add_softmax();
    dlvk::Adam adam2(1e-3);
    m2.build();
    m2.load_weights(out + "/model.dlvk", &adam2);
    m2.save_weights(out + "/model_roundtrip.dlvk", &adam2);
  }

  // ModelTrainer: a few epochs on a learnable synthetic problem.
  {
    at::Generator g2 = at::detail::createCPUGenerator(1);
    at::Tensor xs = at::rand({256, 20}, g2);
    at::Tensor ys = (xs.narrow(1, 0, 1).squeeze(1) > 0.5).to(at::kLong);
    dlvk::Sequential m3(device, 3);
    m3.add_dense(20, 32);
    m3.add_relu();
    m3.add_dense(32, 2);
    m3.add_softmax();
    dlvk::ModelTrainer trainer(&m3);
    trainer.compile(std::make_unique<dlvk::Adam>(1e-2), std::make_unique<dlvk::CrossEntropyLoss>());
    auto hist = trainer.fit(dlvk::Tensor(xs), dlvk::Tensor(ys), 30, 32, 0.25f, false);
    if (hist.size() != 30) return fail("fit history length");
    if (!(hist.back().loss < hist.front().loss)) return fail("training loss did not decrease");
    auto ev = trainer.evaluate(dlvk::Tensor(xs), dlvk::Tensor(ys));
    if (ev.accuracy < 0.8f) return fail("accuracy " + std::to_string(ev.accuracy));
    auto pred = trainer.predict(dlvk::Tensor(xs.narrow(0, 0, 10)));
    if (pred.shape() != std::vector<size_t>({10, 2})) return fail("predict shape");
    std::printf("trainer final loss %.4f acc %.3f\n", hist.back().loss, ev.accuracy);
  }
  // Reference accessor spellings: layer getters / setters, output shapes,
  // optimizer clipping by value and by norm.
  {
    dlvk::Sequential m4(device, 5);
    m4.add_conv2d(1, 4, 3, 1, 1);
    m4.add_batchnorm2d(4);
    m4.add_maxpool2d(2);
    m4.add_flatten();
    m4.add_dense(4 * 4 * 4, 3);
    m4.add_dropout(0.25f);
    m4.build();
    auto* conv = dynamic_cast<dlvk::Conv2DLayer*>(&m4[0]);
    auto* bn = dynamic_cast<dlvk::BatchNormLayer*>(&m4[1]);
    auto* pool = dynamic_cast<dlvk::MaxPool2DLayer*>(&m4[2]);
    auto* dense = dynamic_cast<dlvk::DenseLayer*>(&m4[4]);
    auto* drop = dynamic_cast<dlvk::DropoutLayer*>(&m4[5]);
    if (!conv || !bn || !pool || !dense || !drop) return fail("layer types");
    if (conv->get_weights().shape() != std::vector<size_t>({4, 1, 3, 3}) || conv->get_in_channels() != 1 ||
        conv->get_out_channels() != 4 || conv->get_kernel_height() != 3 || conv->get_kernel_width() != 3)
      return fail("Conv2D accessors");
    if (conv->compute_output_shape({2, 1, 8, 8}) != std::vector<size_t>({2, 4, 8, 8}) ||
        pool->compute_output_shape({2, 4, 8, 8}) != std::vector<size_t>({2, 4, 4, 4}) ||
        pool->get_pool_height() != 2 || pool->get_pool_width() != 2)
      return fail("compute_output_shape");
    bool threw = false;
    try {
      pool->compute_output_shape({1, 1});
    } catch (const std::invalid_argument&) {
      threw = true;
    }
    if (!threw) return fail("compute_output_shape accepted a 2-D shape");
    if (drop->get_dropout_rate() != 0.25f) return fail("get_dropout_rate");
    drop->set_dropout_rate(0.5f);
    if (drop->get_dropout_rate() != 0.5f) return fail("set_dropout_rate");
    bn->set_running_mean(dlvk::Tensor(at::full({4}, 0.5f)));
    if (bn->get_running_mean().to_vector() != std::vector<float>(4, 0.5f)) return fail("BatchNorm running mean");
    if (bn->get_gamma().to_vector() != std::vector<float>(4, 1.f)) return fail("BatchNorm gamma");
    // get_weights() / get_bias() are views of the model's packed weights.
    dense->get_weights().data().zero_();
    dense->get_bias().data().fill_(2.f);
    m4.set_training(false);
    at::Tensor x4 = at::rand({2, 1, 8, 8}, g);
    auto y4 = m4.forward(dlvk::Tensor(x4)).to_vector();
    if (y4 != std::vector<float>(6, 2.f)) return fail("Dense get_weights is not a view");
    // clone(): an independent deep copy
    auto c4 = m4.clone();
    dense->get_bias().data().fill_(3.f);
    if (c4->forward(dlvk::Tensor(x4)).to_vector() != std::vector<float>(6, 2.f)) return fail("clone shares weights");
    if (c4->size() != m4.size() || c4->parameter_count() != m4.parameter_count()) return fail("clone layers");
    auto* relu = dynamic_cast<dlvk::ActivationLayer*>(&model[1]);
    if (!relu || relu->get_activation_type() != dlvk::ActivationType::ReLU) return fail("get_activation_type");

    dlvk::Sequential m5(device, 6);
    m5.add_dense(4, 2);
    m5.build();
    const int64_t n = m5.flat_numel();
    at::Tensor gv = at::linspace(-3.0, 3.0, n).to(m5.master().device());
    dlvk::SGD sgd(1.0);
    sgd.set_grad_clip_value(-1.0, 0.5);
    at::Tensor before = m5.master().clone();
    m5.grad().copy_(gv);
    sgd.step(m5);
    if (!at::allclose(m5.master(), before - gv.clamp(-1.0, 0.5))) return fail("clip by value");
    sgd.disable_grad_clipping();
    sgd.set_grad_clip_norm(1.0);
    before = m5.master().clone();
    m5.grad().copy_(gv);
    sgd.step(m5);
    const float moved = (before - m5.master()).norm().item<float>();
    if (std::fabs(moved - 1.f) > 1e-4f) return fail("clip by norm moved " + std::to_string(moved));
    sgd.disable_grad_clipping();
    before = m5.master().clone();
    m5.grad().copy_(gv);
    sgd.step(m5);
    if (!at::allclose(m5.master(), before - gv)) return fail("disable_grad_clipping");
  }
  std::printf("OK\n");
  return 0;
}
