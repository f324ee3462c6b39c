"""Deployment: dynamic-batching inference engine with per-batch-size CUDA
graphs, HTTP serving, edge packaging and container manifests
(include/dlvk/deployment/inference_deployment.h), and the multi-GPU
trainer API (include/dlvk/deployment/multi_gpu_trainer.h)."""
from .inference import (Config, CrossPlatformDeployment, DeviceConstraints, EdgeDeploymentOptimizer,
                        ModelInferenceEngine, ModelServingServer, ServingConfig, deserialize_tensors,
                        serialize_tensors)
from .multi_gpu import (DeviceInfo, MultiGPUConfig, MultiGPUDeviceManager, MultiGPUTrainer, RingAllReduce,
                        TrainingStats, VulkanCommunicationBackend)
