"""Loader of the native extension `dlvk_b200._C`.

The extension is built ahead of time (``python -m dlvk_b200._build`` or
``__graft_entry__.build()``) into the package directory and imported from
there.  When a CUDA device is present the extension is mandatory: every GPU
op dispatches into it and there is no silent PyTorch fallback.
"""
from __future__ import annotations

import importlib
import os

_C = None
_err = None


def load(build_if_missing: bool = True):
    """Import (building first if needed) and return the `_C` module."""
    global _C, _err
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("dlvk_b200._C")
        return _C
    except ImportError as exc:  # not built yet
        _err = exc
    if build_if_missing and os.environ.get("DLVK_NO_BUILD", "0") != "1":
        from . import _build

        _build.build()
        _C = importlib.import_module("dlvk_b200._C")
        return _C
    raise ImportError(f"dlvk_b200 native extension is not built: {_err}")


def C():
    """The native module; raises loudly if it cannot be loaded."""
    return _C if _C is not None else load()


def available() -> bool:
    try:
        load(build_if_missing=False)
        return True
    except ImportError:
        return False
