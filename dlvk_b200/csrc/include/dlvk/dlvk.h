// Umbrella header of the dlvk_b200 C++ API (link libdlvk_b200.so).
#pragma once
#include "dlvk/core/cuda_device.h"
#include "dlvk/layers/layers.h"
#include "dlvk/loss/loss_functions.h"
#include "dlvk/model/model.h"
#include "dlvk/optimizers/optimizers.h"
#include "dlvk/tensor/tensor.h"
#include "dlvk/tensor/tensor_ops_static.h"
