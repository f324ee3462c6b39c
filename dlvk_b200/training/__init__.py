"""Training: captured training step, Keras-style trainer and callbacks,
DataLoader-driven Trainer, mixed precision, regularisation, advanced
trainer / schedulers / search, persistence (include/dlvk/training/*,
include/dlvk/model/*)."""
from .step import TrainStep
from .callbacks import (CSVLogger, EarlyStopping, EarlyStoppingCallback, LambdaCallback, ModelCheckpoint,
                        ProgressCallback, ReduceLROnPlateau, TrainingCallback, TrainingMetrics)
from .model_trainer import ModelTrainer
from .trainer import Trainer, create_trainer, make_loss, make_optimizer
from .mixed_precision import (AutocastContext, GradientScaler, MixedPrecisionContext, MixedPrecisionTrainer,
                              PrecisionMode)
from .regularization import (AdvancedDropout, ElasticNetRegularizer, L1Regularizer, L2Regularizer,
                             RegularizationManager, RegularizationType, Regularizer, WeightDecayRegularizer,
                             create_comprehensive_regularization, create_elastic_net, create_l2_regularization,
                             create_weight_decay)
from .advanced import (AdvancedTrainer, AdvancedTrainingConfig, CosineAnnealingScheduler, CyclicScheduler,
                       ExponentialScheduler, HyperparameterConfig, HyperparameterRange, HyperparameterResult,
                       LearningRateScheduler, LRScheduleType, OneCycleScheduler, ReduceOnPlateauScheduler,
                       StepDecayScheduler, TrainingStatistics, create_advanced_trainer, random_search)
from . import persistence
from .persistence import (CheckpointData, ModelCheckpointCallback, ModelSerializer, ModelVersioning,
                          SerializationFormat)
from .persistence import ModelCheckpoint as CheckpointManager
from .persistence import create_checkpoint_callback, create_versioning_system
from types import SimpleNamespace as _NS

# The reference's namespace persistence_factory (model_persistence.h:362-381).
persistence_factory = _NS(create_checkpoint_callback=create_checkpoint_callback,
                          create_versioning_system=create_versioning_system)
