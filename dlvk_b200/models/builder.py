"""Rebuild a Sequential model from its architecture description (the
per-layer dicts `Sequential.architecture()` stores in every `.dlvk` v2
file's metadata), so a checkpoint can be loaded without the code that
built the model (the reference's `ModelSerializer::load_binary` returned
nullptr, src/training/model_persistence.cpp:93-124)."""
from __future__ import annotations

from typing import List

from . import layers as L


def layer_from_config(d: dict) -> L.ModernLayer:
    t = d["type"]
    g = d.get
    if t == "Dense":
        return L.DenseLayer(d["input_size"], d["output_size"], g("use_bias", True), g("activation"))
    if t == "Conv2D":
        return L.Conv2DLayer(d["in_channels"], d["out_channels"], d["kernel_size"], g("stride", 1), g("padding", 0),
                             g("activation"), g("use_bias", True))
    if t == "MaxPool2D":
        return L.MaxPool2DLayer(d["pool_size"], g("stride", 0))
    if t == "AvgPool2D":
        return L.AvgPool2DLayer(d["pool_size"], g("stride", 0), g("padding", 0))
    if t == "BatchNorm1D":
        return L.BatchNorm1DLayer(d["num_features"], g("momentum", 0.1), g("eps", 1e-5))
    if t == "BatchNorm2D":
        return L.BatchNorm2DLayer(d["num_features"], g("momentum", 0.1), g("eps", 1e-5))
    if t == "Dropout":
        return L.DropoutLayer(d["rate"])
    if t == "Activation":
        return L.ActivationLayer(d["activation"])
    if t == "Flatten":
        return L.FlattenLayer()
    if t == "Embedding":
        return L.EmbeddingLayer(d["num_embeddings"], d["embedding_dim"])
    if t == "LayerNorm":
        return L.LayerNormLayer(d["normalized_shape"], g("eps", 1e-5))
    if t == "MultiHeadAttention":
        return L.MultiHeadAttentionLayer(d["embed_dim"], d["num_heads"], residual=g("residual", False))
    if t == "PositionalEncoding":
        return L.PositionalEncodingLayer(d["d_model"], g("max_len", 5000))
    if t == "Residual":
        return L.ResidualLayer(layer_from_config(d["inner"]))
    if t == "GlobalAvgPool":
        return L.GlobalAvgPoolLayer()
    if t == "TransformerEncoder":
        return L.TransformerEncoderLayer(d["d_model"], d["nhead"], g("dim_feedforward", 2048))
    if t == "GroupNorm":
        return L.GroupNormLayer(d["num_groups"], d["num_channels"], g("eps", 1e-5))
    if t in ("RNN", "LSTM", "GRU"):
        cls = {"RNN": L.RNNLayer, "LSTM": L.LSTMLayer, "GRU": L.GRULayer}[t]
        return cls(d["input_size"], d["hidden_size"], g("return_sequences", True), g("reverse", False),
                   g("use_bias", True))
    if t == "Bidirectional":
        return L.BidirectionalRNN(d["cell"], d["input_size"], d["hidden_size"], g("return_sequences", True))
    raise ValueError(f"unknown layer type '{t}' in architecture")


def model_from_architecture(arch: List[dict], device=None, dtype="fp32"):
    from .sequential import Sequential

    m = Sequential(device, dtype)
    for d in arch:
        m.add(layer_from_config(d))
    return m.build()


def load_model_file(path: str, device=None, dtype=None, optimizer=None):
    """Rebuild the model stored in a `.dlvk` v2 file and load its weights."""
    from ..utils import dlvk_io

    _, variant, meta, _ = dlvk_io.load(path)
    if "architecture" not in meta:
        raise ValueError(f"{path}: no architecture in the file's metadata ({variant})")
    m = model_from_architecture(meta["architecture"], device, dtype or meta.get("compute_dtype", "fp32"))
    m.load_weights(path, optimizer=optimizer)
    return m
