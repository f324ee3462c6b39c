"""Layers, Sequential and the model zoo of the benchmark configurations."""
