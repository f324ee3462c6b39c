"""dlvk_b200: a B200-native (sm_100a) deep-learning framework with the
capabilities and public API of DLVK.

Hot ops run as hand-written sm_100a kernels (tcgen05/TMEM/TMA GEMMs, fused
norms, softmax-cross-entropy, optimizers, fused all-reduce + optimizer) from
the in-tree extension `dlvk_b200._C`; tensors, autograd bookkeeping and the
training loop sit on PyTorch.
"""
__version__ = "0.1.0"

from . import runtime
from .runtime import CudaDevice, get_device
from .tensor import Tensor, TensorOps, TensorOpsStatic, DataType
from .models.layers import (ModernLayer, Layer, LayerInfo, ActivationType, DenseLayer, Conv2DLayer, MaxPool2DLayer,
                            AvgPool2DLayer, BatchNorm1DLayer, BatchNorm2DLayer, DropoutLayer, ActivationLayer,
                            FlattenLayer, EmbeddingLayer, LayerNormLayer, MultiHeadAttentionLayer,
                            TransformerEncoderLayer, PositionalEncodingLayer, GroupNormLayer, ResidualLayer,
                            GlobalAvgPoolLayer, manual_seed)
from .models.sequential import Model, Sequential
from .models.params import Parameter, ParamStore
from .optim import (Optimizer, SGD, Adam, RMSprop, GradientClipping, LRScheduler, StepLRScheduler,
                    ExponentialLRScheduler, CosineAnnealingLRScheduler, LinearLRScheduler)
from .losses import LossFunction, CrossEntropyLoss, MeanSquaredError, BinaryCrossEntropyLoss, MSELoss, BCELoss

# The reference spells the device class VulkanDevice; this framework's device
# runtime is CUDA.
VulkanDevice = CudaDevice
