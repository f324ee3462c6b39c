"""Model export / import: DLVK, ONNX, GGUF v3, SafeTensors, HDF5 (with
h5py) (include/dlvk/export/model_export.h)."""
from .model_export import (DLVKExporter, GGUFExporter, HDF5Exporter, ModelExporter, ModelExportManager,
                           ModelFormat, ModelMetadata, ONNXExporter, SafeTensorsExporter, TensorInfo,
                           create_export_manager, extract_tensors)

__all__ = ["DLVKExporter", "GGUFExporter", "HDF5Exporter", "ModelExporter", "ModelExportManager", "ModelFormat",
           "ModelMetadata", "ONNXExporter", "SafeTensorsExporter", "TensorInfo", "create_export_manager",
           "extract_tensors"]
