"""Utilities: .dlvk I/O, tracing, configuration."""
