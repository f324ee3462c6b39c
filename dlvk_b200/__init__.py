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
from .losses import (LossFunction, CrossEntropyLoss, MeanSquaredError, BinaryCrossEntropyLoss, MSELoss, BCELoss,
                     LossOpsGPU)

# The reference spells the device class VulkanDevice; this framework's device
# runtime is CUDA.
VulkanDevice = CudaDevice

from .models.layers import (RNNLayer, LSTMLayer, GRULayer, BidirectionalRNN, BiLSTM, BiGRU, BiRNN, ConvLayer)
from .models.builder import model_from_architecture, load_model_file
from .training import (TrainStep, ModelTrainer, Trainer, create_trainer, TrainingMetrics, TrainingCallback,
                       ProgressCallback, ModelCheckpoint, EarlyStopping, EarlyStoppingCallback, ReduceLROnPlateau,
                       CSVLogger, PrecisionMode, GradientScaler, MixedPrecisionContext, AutocastContext,
                       MixedPrecisionTrainer, RegularizationManager, L1Regularizer, L2Regularizer,
                       ElasticNetRegularizer, WeightDecayRegularizer, AdvancedDropout, AdvancedTrainer,
                       AdvancedTrainingConfig, create_advanced_trainer, ModelSerializer, ModelVersioning,
                       CheckpointManager)
from . import data, export, deployment, optimization, training, parallel
from .data import DataLoader, MnistDataset, Dataset, TransformDataset
from .export import ModelExportManager, ModelFormat
from .optimization.model_optimizer import ModelOptimizer, QuantizationConfig, PruningConfig
from .deployment import ModelInferenceEngine, ModelServingServer, MultiGPUTrainer, MultiGPUDeviceManager
