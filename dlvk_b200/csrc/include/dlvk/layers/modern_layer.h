// C++ API: the layer interface (include/dlvk/layers/modern_layer.h:20-80 of
// the reference) plus what the framework needs from a layer: its trainable
// parameters (packed by Sequential into flat buffers, like the Python
// package's ParamStore) and its persistent buffers.
#pragma once
#include <ATen/ATen.h>

#include <fstream>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "dlvk/tensor/tensor.h"

namespace dlvk {

class Optimizer;

struct LayerInfo {
  std::string type;
  std::string output_shape_str;
  size_t parameter_count = 0;
  bool trainable = false;
};

// One trainable tensor.  After Sequential::build() `master` and `grad` are
// views into the model's flat fp32 buffers.
struct Parameter {
  std::string name;
  std::vector<int64_t> shape;
  at::Tensor master;  // fp32 weights
  at::Tensor grad;    // fp32 gradient
  bool fresh = true;  // the next gradient write overwrites instead of adding
  int64_t offset = -1;
  const void* store = nullptr;  // the Sequential whose flat buffers hold it
  int64_t numel() const;
  // True if the next gradient write must accumulate; marks the gradient written.
  bool take_accumulate();
};

class ModernLayer {
 public:
  ModernLayer() = default;
  // Copies deep-copy the parameters (unpacked from any model's buffers).
  ModernLayer(const ModernLayer& other);
  ModernLayer& operator=(const ModernLayer&) = delete;
  virtual ~ModernLayer() = default;

  virtual Tensor forward(const Tensor& input) = 0;
  virtual Tensor backward(const Tensor& grad_output) = 0;
  virtual std::unique_ptr<ModernLayer> clone() const = 0;

  // Applies `optimizer` to this layer's parameters only.
  virtual void update_parameters(Optimizer& optimizer);
  virtual void set_training(bool training) { training_ = training; }
  virtual LayerInfo get_layer_info() const;
  // u32 tensor count, then per tensor u64 byte count + raw fp32 values
  // (the Python package's per-layer stream format).
  virtual void save_weights(std::ofstream& file) const;
  virtual void load_weights(std::ifstream& file);

  // Framework hooks.
  virtual std::string type_name() const = 0;
  // Architecture entry of the `.dlvk` metadata, keys sorted (JSON object).
  virtual std::string config_json() const;
  std::vector<Parameter*> parameters();
  // Parameters and persistent buffers, with their `.dlvk` record names.
  virtual std::vector<std::pair<std::string, at::Tensor*>> state_tensors();
  size_t parameter_count() const;
  bool training() const { return training_; }
  std::vector<int64_t> output_shape;
  // False for the first layer of a model: its input needs no gradient, so
  // backward() skips the dX computation and returns an undefined tensor.
  bool need_input_grad = true;

 protected:
  Parameter& add_param(const std::string& name, at::Tensor init);
  virtual std::vector<std::pair<std::string, at::Tensor*>> buffers() { return {}; }
  std::vector<std::unique_ptr<Parameter>> params_;
  bool training_ = true;
};

}  // namespace dlvk
